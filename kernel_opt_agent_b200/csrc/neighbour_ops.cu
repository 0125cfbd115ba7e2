// neighbour_ops.cu -- the harness's other registered row-wise ops, as further plugins behind the
// same C ABI: RMS norm, SwiGLU with FP8 input quantisation, and partial rotary embedding of a
// packed QKV tensor.  All three are HBM-bound (a few flops per byte), so each kernel reads its
// input once with 16-byte vector accesses and writes its outputs once; no shared-memory tiling,
// no tensor cores, no waits.
//
//  * rms_norm (references/rms_norm.py:6-10):  out = x / sqrt(mean(x^2) + eps) * weight, fp32
//    arithmetic, result in x's type (bf16 or fp16).  One warp per row, two passes over the row
//    (the second hits L1: rows are at most a few KB).
//  * swiglu_input_quant (references/swiglu_input_quant.py:6-30):  out = x0 * silu(x1) (x = [x0|x1],
//    x1 in fp32, product cast to bf16); x_fp8 = e4m3(bf16(x * bf16(1/scale))) per 128-column block
//    with scale = max(amax|block|, eps) / 448, stored with x_scale as [n_blocks, M].  One warp per
//    (row, 128-column block): lane l holds 4 columns.
//  * qkv_part_rope (references/qkv_part_rope.py:6-45):  a copy of qkv [B,S,H,D] whose first
//    q_heads + kv_heads heads have their last rope_dim = D - nope_dim columns rotated by (cos, sin)
//    of the token's position (pairs (i, i + rope_dim/2)); the value heads pass through.  One CTA
//    per (batch, token) row of H*D elements.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "host_common.h"

namespace tokmix {
namespace ops {

// ------------------------------------------------------------------------------------ RMS norm
template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half x) {
  return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_f<__half>(float x) {
  return __float2half_rn(x);
}

template <typename T>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* x, const T* w, T* out, int rows, int n, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // warp-uniform
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * n);
  const int nvec = n / 8;  // 8 elements per 16-byte vector
  float ss = 0.0f;
  for (int i = lane; i < nvec; i += 32) {
    const uint4 v = xr[i];
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = to_f<T>(e[j]);
      ss += f * f;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rms = sqrtf(ss / static_cast<float>(n) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * n);
  for (int i = lane; i < nvec; i += 32) {
    const uint4 v = xr[i];
    const uint4 wv = wr[i];
    const T* e = reinterpret_cast<const T*>(&v);
    const T* we = reinterpret_cast<const T*>(&wv);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) oe[j] = from_f<T>(to_f<T>(e[j]) / rms * to_f<T>(we[j]));
    orow[i] = o;
  }
}

// ---------------------------------------------------------------------- SwiGLU + FP8 quantisation
// One warp per (row, 128-column block b of x); blocks b < n/128 also produce out's block b.
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const __nv_bfloat16* x, __nv_bfloat16* out,
                                                           __nv_fp8_e4m3* xq, float* xscale, int m, int n, float eps) {
  const int nb2 = (2 * n) / 128;  // blocks per row of x
  const long long item = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= static_cast<long long>(m) * nb2) return;  // warp-uniform
  const int row = static_cast<int>(item / nb2);
  const int blk = static_cast<int>(item - static_cast<long long>(row) * nb2);
  const int col = blk * 128 + 4 * lane;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * 2 * n;
  const uint2 raw = *reinterpret_cast<const uint2*>(xr + col);
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
  // block amax -> scale, then x * bf16(1/scale) in bf16, then e4m3 (saturating)
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(e[j])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = fmaxf(amax, eps) / 448.0f;
  const __nv_bfloat16 inv = __float2bfloat16_rn(1.0f / scale);
  uint32_t q4 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat16 prod = __hmul(e[j], inv);
    const __nv_fp8_storage_t q8 = __nv_cvt_float_to_fp8(__bfloat162float(prod), __NV_SATFINITE, __NV_E4M3);
    q4 |= static_cast<uint32_t>(q8) << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(xq) + static_cast<size_t>(row) * 2 * n + col) = q4;
  if (lane == 0) xscale[static_cast<size_t>(blk) * m + row] = scale;
  if (blk < n / 128) {  // out block: x0 * (x1 * sigmoid(x1)) in fp32, cast to bf16
    const uint2 raw1 = *reinterpret_cast<const uint2*>(xr + n + col);
    const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&raw1);
    __nv_bfloat16 o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x1 = __bfloat162float(e1[j]);
      o[j] = __float2bfloat16_rn(__bfloat162float(e[j]) * (x1 * (1.0f / (1.0f + expf(-x1)))));
    }
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(row) * n + col) = *reinterpret_cast<const uint2*>(o);
  }
}

// -------------------------------------------------------------------------- partial rotary QKV
// One CTA per (batch, token) row: heads x head_dim elements.  Thread i < rows_pairs rotates one
// (i, i + half) pair of a q/k head; every other element is copied in 16-byte vectors.
__global__ void __launch_bounds__(256) qkv_part_rope_kernel(const __nv_bfloat16* qkv, const float* cosv,
                                                            const float* sinv, __nv_bfloat16* out, int seq, int heads,
                                                            int head_dim, int nope, int rot_heads, float sin_sign) {
  const long long rowi = blockIdx.x;  // batch * seq + s
  const int s = static_cast<int>(rowi % seq);
  const int half = (head_dim - nope) / 2;
  const size_t base = static_cast<size_t>(rowi) * heads * head_dim;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + base);
  uint4* dst = reinterpret_cast<uint4*>(out + base);
  const int nvec = heads * head_dim / 8;
  const int nope_vec = nope / 8, dvec = head_dim / 8;
  // copy: value heads entirely, and the nope columns of the rotated heads
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const int h = i / dvec, c = i - h * dvec;
    if (h >= rot_heads || c < nope_vec) dst[i] = src[i];
  }
  // rotate: pair (nope + j, nope + half + j) of head h
  for (int i = threadIdx.x; i < rot_heads * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    const size_t o0 = base + static_cast<size_t>(h) * head_dim + nope + j;
    const float x0 = __bfloat162float(qkv[o0]);
    const float x1 = __bfloat162float(qkv[o0 + half]);
    const float c = cosv[static_cast<size_t>(s) * half + j];
    const float sn = sin_sign * sinv[static_cast<size_t>(s) * half + j];
    out[o0] = __float2bfloat16_rn(x0 * c - x1 * sn);
    out[o0 + half] = __float2bfloat16_rn(x0 * sn + x1 * c);
  }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace ops
}  // namespace tokmix

extern "C" int tokmix_rms_norm(const void* x, const void* weight, void* out, int rows, int n, int dtype, float eps,
                               void* stream) {
  using namespace tokmix;
  using namespace tokmix::ops;
  if (rows < 0 || n <= 0) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_rms_norm: bad shape (%d, %d)", rows, n);
  if (n % 8 != 0) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_rms_norm: row length must be a multiple of 8");
  if (dtype != TOKMIX_DTYPE_BF16 && dtype != TOKMIX_DTYPE_FP16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_rms_norm: bf16 or fp16 only (dtype %d)", dtype);
  if (!(eps >= 0.0f) || !std::isfinite(eps)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_rms_norm: bad eps");
  if (rows == 0) return TOKMIX_OK;
  if (!x || !weight || !out) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_rms_norm: null pointer argument");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_rms_norm: tensors must be 16-byte aligned");
  if (const int rc = check_device()) return rc;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TOKMIX_DTYPE_BF16)
    rms_norm_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                          static_cast<const __nv_bfloat16*>(weight),
                                                          static_cast<__nv_bfloat16*>(out), rows, n, eps);
  else
    rms_norm_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(weight),
                                                   static_cast<__half*>(out), rows, n, eps);
  return check_launch("tokmix_rms_norm");
}

extern "C" int tokmix_swiglu_input_quant(const void* x, void* out, void* x_fp8, float* x_scale, int m, int n,
                                         float eps, void* stream) {
  using namespace tokmix;
  using namespace tokmix::ops;
  if (m < 0 || n <= 0) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_swiglu_input_quant: bad shape (%d, %d)", m, n);
  if (n % 128 != 0)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_swiglu_input_quant: n must be a multiple of 128 (got %d)", n);
  if (!(eps > 0.0f) || !std::isfinite(eps))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_swiglu_input_quant: eps must be finite and positive");
  if (m == 0) return TOKMIX_OK;
  if (!x || !out || !x_fp8 || !x_scale)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_swiglu_input_quant: null pointer argument");
  if (!aligned16(x) || !aligned16(out) || !aligned16(x_fp8) || !aligned16(x_scale))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_swiglu_input_quant: tensors must be 16-byte aligned");
  const long long items = static_cast<long long>(m) * (2 * n / 128);
  if ((items + 7) / 8 > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_swiglu_input_quant: too large");
  if (const int rc = check_device()) return rc;
  swiglu_quant_kernel<<<static_cast<unsigned>((items + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), static_cast<__nv_fp8_e4m3*>(x_fp8),
      x_scale, m, n, eps);
  return check_launch("tokmix_swiglu_input_quant");
}

extern "C" int tokmix_qkv_part_rope(const void* qkv, const float* cos, const float* sin, void* out, int batch, int seq,
                                    int heads, int head_dim, int q_heads, int kv_heads, int nope_dim, int negative_sin,
                                    void* stream) {
  using namespace tokmix;
  using namespace tokmix::ops;
  if (batch < 0 || seq < 0 || heads <= 0 || head_dim <= 0 || q_heads < 0 || kv_heads < 0 || nope_dim < 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_qkv_part_rope: negative size");
  if (q_heads + kv_heads > heads)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_qkv_part_rope: q_heads + kv_heads exceeds the head count");
  if (head_dim % 8 != 0 || nope_dim % 8 != 0 || nope_dim > head_dim || (head_dim - nope_dim) % 2 != 0)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_qkv_part_rope: head_dim and nope_dim must be multiples of 8");
  if (batch == 0 || seq == 0) return TOKMIX_OK;
  if (!qkv || !out || (head_dim > nope_dim && (!cos || !sin)))  // no table is read when nothing rotates
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_qkv_part_rope: null pointer");
  if (!aligned16(qkv) || !aligned16(out))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_qkv_part_rope: tensors must be 16-byte aligned");
  const long long rows = static_cast<long long>(batch) * seq;
  if (rows > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_qkv_part_rope: too many rows");
  if (const int rc = check_device()) return rc;
  qkv_part_rope_kernel<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), cos, sin, static_cast<__nv_bfloat16*>(out), seq, heads, head_dim,
      nope_dim, q_heads + kv_heads, negative_sin ? -1.0f : 1.0f);
  return check_launch("tokmix_qkv_part_rope");
}
