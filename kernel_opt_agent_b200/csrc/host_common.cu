// host_common.cu -- error reporting, tensor-map encoding and device queries for the C ABI.
#include "host_common.h"

#include <cmath>

#include <mutex>
#include <set>
#include <utility>

namespace tokmix {

namespace {
thread_local std::string g_last_error;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TOKMIX_OK;
  return fail(TOKMIX_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
    return false;
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, bx, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    return false;
  }
  return true;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

bool ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<std::pair<const void*, int>, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(std::make_pair(func, dev), bytes);
  if (done.count(key)) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  done.insert(key);
  return true;
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TOKMIX_ERR_DEVICE, "no CUDA device");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(TOKMIX_ERR_DEVICE, "libtokmix is built for sm_100a (B200); device %d is sm_%d%d", dev, major, minor);
  return TOKMIX_OK;
}

}  // namespace tokmix

namespace tokmix {

int check_stage1(const char* who, const tokmix_gdn_stage1* s1, bool needs_k_normed) {
  if (s1 == nullptr) return TOKMIX_OK;
  if (stage1_gates(s1) && (!s1->b || !s1->a_log || !s1->dt_bias ||
                           (s1->dtype != TOKMIX_DTYPE_BF16 && s1->dtype != TOKMIX_DTYPE_FP32)))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: gates need a, b, a_log, dt_bias and a bf16 or fp32 dtype", who);
  if (stage1_l2norm(s1)) {
    if (!(s1->l2norm_eps > 0.0f) || !std::isfinite(s1->l2norm_eps))
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: l2norm_eps must be positive and finite", who);
    if (needs_k_normed && (s1->k_normed == nullptr || reinterpret_cast<uintptr_t>(s1->k_normed) % 16 != 0))
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: qk_l2norm needs a 16-byte aligned k_normed buffer", who);
  }
  return TOKMIX_OK;
}

}  // namespace tokmix

extern "C" const char* tokmix_last_error(void) { return tokmix::g_last_error.c_str(); }

extern "C" const char* tokmix_version(void) { return "tokmix 0.1.0 sm_100a"; }
