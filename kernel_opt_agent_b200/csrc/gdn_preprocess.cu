// gdn_preprocess.cu -- the steps before the GDN kernels that the reference leaves to its caller
// (kernels/qwen35moe_gdn_prefill.py:107-136 takes normalised q/k and ready g, beta):
//
//  * l2norm_rows_kernel (the qk_l2norm option): y[r] = x[r] / sqrt(sum_i x[r][i]^2 + eps), fp32
//    arithmetic, bf16 result -- the GDN kernels' operand type, so for fp32 inputs it replaces the
//    plain conversion pass.  Rows of 128, input bf16 or fp32.  One warp per row (lane l holds
//    elements 4l .. 4l+3), a warp butterfly for the sum of squares; HBM-bound.
//  * gdn_gates_kernel (the gates option): the Qwen3.5 gated-delta-net gates from the raw
//    projections a, b [tokens, heads_v] and the per-head parameters A_log, dt_bias [heads_v]:
//        g = -exp(A_log[h]) softplus(a + dt_bias[h]),   beta = sigmoid(b)     (fp32)
//    One thread per (token, head).  g and beta are T x Hv floats, so this pass costs about as much
//    as reading them once more -- well under a microsecond at the benchmark shapes.
// No shared memory and no waits in either kernel.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "gdn_common.cuh"
#include "host_common.h"

namespace tokmix {
namespace preprocess {

constexpr int kDim = 128;
constexpr int kWarps = 8;

template <typename T>
__device__ __forceinline__ void load4(const T* row, int lane, float (&f)[4]);

template <>
__device__ __forceinline__ void load4<float>(const float* row, int lane, float (&f)[4]) {
  const float4 v = __ldcs(reinterpret_cast<const float4*>(row) + lane);
  f[0] = v.x;
  f[1] = v.y;
  f[2] = v.z;
  f[3] = v.w;
}

template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* row, int lane, float (&f)[4]) {
  const uint2 w = __ldcs(reinterpret_cast<const uint2*>(row) + lane);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) l2norm_rows_kernel(const T* x, __nv_bfloat16* y, long long rows,
                                                                  float eps) {
  const long long r = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;  // whole warps leave together (r is warp-uniform)
  float f[4];
  load4<T>(x + r * kDim, lane, f);
  // the order of the sum is fixed (gdn_common.cuh, l2norm_row_sw128 forms it the same way inside
  // the GDN kernels): 4 consecutive elements per lane, then an XOR butterfly
  float ss = gdn::sumsq4(f[0], f[1], f[2], f[3]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const float inv = rsqrtf(ss + eps);
  const __nv_bfloat162 a = __floats2bfloat162_rn(f[0] * inv, f[1] * inv);
  const __nv_bfloat162 b = __floats2bfloat162_rn(f[2] * inv, f[3] * inv);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&a);
  w.y = *reinterpret_cast<const uint32_t*>(&b);
  __stcs(reinterpret_cast<uint2*>(y + r * kDim) + lane, w);
}

template <typename T>
__global__ void __launch_bounds__(256) gdn_gates_kernel(const T* a, const T* b, const float* a_log,
                                                        const float* dt_bias, float* g, float* beta, long long n,
                                                        int hv) {
  const long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n) return;
  const int h = static_cast<int>(i % hv);
  // the same arithmetic as the GDN kernels' own gate loads (gdn_common.cuh: load_gates)
  gdn::GateSource gs{a, b, a_log, dt_bias, sizeof(T) == 2 ? 1 : 0};
  float gv, bv;
  gdn::load_gates(nullptr, nullptr, gs, static_cast<size_t>(i), h, gv, bv);
  g[i] = gv;
  beta[i] = bv;
}

}  // namespace preprocess
}  // namespace tokmix

extern "C" int tokmix_gdn_gates(const void* a, const void* b, int ab_dtype, const float* a_log, const float* dt_bias,
                                float* g, float* beta, long long tokens, int heads_v, void* stream) {
  using namespace tokmix;
  using namespace tokmix::preprocess;
  if (tokens < 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_gates: negative token count or non-positive head count");
  if (ab_dtype != TOKMIX_DTYPE_BF16 && ab_dtype != TOKMIX_DTYPE_FP32)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_gates: unknown input dtype %d", ab_dtype);
  if (tokens == 0) return TOKMIX_OK;
  if (!a || !b || !a_log || !dt_bias || !g || !beta)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_gates: null pointer argument");
  const long long n = tokens * heads_v;
  const long long blocks = (n + 255) / 256;
  if (blocks > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_gates: too many elements");
  if (const int rc = check_device()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ab_dtype == TOKMIX_DTYPE_FP32)
    gdn_gates_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const float*>(a), static_cast<const float*>(b), a_log, dt_bias, g, beta, n, heads_v);
  else
    gdn_gates_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), a_log, dt_bias, g, beta, n,
        heads_v);
  return check_launch("tokmix_gdn_gates");
}

extern "C" int tokmix_l2norm_rows(const void* x, int x_dtype, void* y, long long rows, int dim, float eps,
                                  void* stream) {
  using namespace tokmix;
  using namespace tokmix::preprocess;
  if (rows < 0) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_l2norm_rows: negative row count");
  if (dim != kDim) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_l2norm_rows: rows of 128 only (got %d)", dim);
  if (x_dtype != TOKMIX_DTYPE_BF16 && x_dtype != TOKMIX_DTYPE_FP32)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_l2norm_rows: unknown input dtype %d", x_dtype);
  if (!(eps >= 0.0f) || !std::isfinite(eps))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_l2norm_rows: eps must be finite and non-negative");
  if (rows == 0) return TOKMIX_OK;
  if (!x || !y) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_l2norm_rows: null pointer argument");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(y) % 16 != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_l2norm_rows: tensors must be 16-byte aligned");
  const long long blocks = (rows + kWarps - 1) / kWarps;
  if (blocks > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_l2norm_rows: too many rows");
  if (const int rc = check_device()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == TOKMIX_DTYPE_FP32)
    l2norm_rows_kernel<float><<<static_cast<unsigned>(blocks), kWarps * 32, 0, s>>>(
        static_cast<const float*>(x), static_cast<__nv_bfloat16*>(y), rows, eps);
  else
    l2norm_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), kWarps * 32, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), rows, eps);
  return check_launch("tokmix_l2norm_rows");
}
