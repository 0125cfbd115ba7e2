// neighbour_ops.cu -- the harness's other registered row-wise ops, as further plugins behind the
// same C ABI: RMS norm, SwiGLU with FP8 input quantisation, and partial rotary embedding of a
// packed QKV tensor.  All three are HBM-bound (a few flops per byte), so each kernel reads its
// input once with 16-byte vector accesses (streaming: evict-first) and writes its outputs once;
// no shared-memory tiling, no tensor cores, no waits.
//
//  * rms_norm (references/rms_norm.py:6-10):  out = x / sqrt(mean(x^2) + eps) * weight, fp32
//    arithmetic, result in x's type (bf16 or fp16).  One warp per row holding the whole row in
//    registers (rows up to 8192 elements), so x crosses HBM once; longer rows take two passes.
//  * swiglu_input_quant (references/swiglu_input_quant.py:6-30):  out = x0 * silu(x1) (x = [x0|x1],
//    x1 in fp32, product cast to bf16); x_fp8 = e4m3(bf16(x * bf16(1/scale))) per 128-column block
//    with scale = max(amax|block|, eps) * fp32(1/448), stored with x_scale as [n_blocks, M].  Half
//    a warp per unit (row, block b): block b of x0 and block b of x1 (lane = 8 columns of each),
//    which is exactly what out's block b needs, so x is read once.
//  * qkv_part_rope (references/qkv_part_rope.py:6-45):  a copy of qkv [B,S,H,D] whose first
//    q_heads + kv_heads heads have their last rope_dim = D - nope_dim columns rotated by (cos, sin)
//    of the token's position (pairs (i, i + rope_dim/2)); the value heads pass through.  One warp
//    per (token, 4 heads), lane = one 16-byte vector of a head; a rotated vector takes its partner
//    from the partner's lane by shuffle.  The products and sums are rounded one by one (no fused
//    multiply-add), as the checker's tensor operations round them.  Shapes outside that layout
//    (head_dim > 256 or rope_dim not a multiple of 16) take a per-row kernel.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <typename T>
__device__ __forceinline__ uint4 rms_scale_vec(uint4 v, uint4 wv, float inv) {
  const T* e = reinterpret_cast<const T*>(&v);
  const T* we = reinterpret_cast<const T*>(&wv);
  uint4 o;
  T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) oe[j] = from_f<T>(to_f<T>(e[j]) * inv * to_f<T>(we[j]));
  return o;
}

// Sum of squares of 8 packed values.  The widening is written in inline assembly so that the
// compiler cannot share it with the output pass's conversions: otherwise it keeps all of a row's
// floats alive between the passes (twice the registers of the packed row, a quarter of the warps).
__device__ __forceinline__ void widen2(uint32_t w, float& lo, float& hi, __nv_bfloat16) {
  asm("prmt.b32 %0, %2, 0, 0x1044;\n\tprmt.b32 %1, %2, 0, 0x3244;" : "=f"(lo), "=f"(hi) : "r"(w));
}
__device__ __forceinline__ void widen2(uint32_t w, float& lo, float& hi, __half) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(w));
}

template <typename T>
__device__ __forceinline__ float sum_sq(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float lo, hi;
    widen2(w[j], lo, hi, T());
    ss += lo * lo;
    ss += hi * hi;
  }
  return ss;
}

// Persistent CTAs of 8 warps; each warp takes rows row0, row0 + 8 * gridDim.x, ... and holds the
// row in registers: lane l owns 16-byte vectors l, l + 32, ... (VPL of them).  The weight vector
// is staged once per CTA in shared memory, so only the row's own vectors occupy registers.
template <typename T, int VPL>
__global__ void __launch_bounds__(256) rms_norm_reg_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                           T* __restrict__ out, int rows, int n, float eps) {
  __shared__ uint4 wsm[32 * VPL];
  const int nvec = n / 8;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) wsm[i] = __ldg(reinterpret_cast<const uint4*>(w) + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += gridDim.x * 8) {  // warp-uniform
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * n);
    uint4 v[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int i = lane + 32 * k;
      v[k] = i < nvec ? __ldcs(xr + i) : make_uint4(0u, 0u, 0u, 0u);
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) ss += sum_sq<T>(v[k]);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    uint4* orow = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * n);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int i = lane + 32 * k;
      if (i < nvec) __stcs(orow + i, rms_scale_vec<T>(v[k], wsm[i], inv));
    }
  }
}

// Rows longer than 8192 elements: two passes over the row, one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                       T* __restrict__ out, int rows, int n, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // warp-uniform
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * n);
  const int nvec = n / 8;
  float ss = 0.0f;
  for (int i = lane; i < nvec; i += 32) ss += sum_sq<T>(xr[i]);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * n);
  for (int i = lane; i < nvec; i += 32) __stcs(orow + i, rms_scale_vec<T>(__ldcs(xr + i), __ldg(wr + i), inv));
}

template <typename T>
void launch_rms_norm(const T* x, const T* w, T* out, int rows, int n, float eps, int sms, cudaStream_t s) {
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  const unsigned persistent = std::min<unsigned>(blocks, static_cast<unsigned>(sms) * 4);
  const int per_lane = (n / 8 + 31) / 32;
#define TOKMIX_RMS_CASE(V) \
  if (per_lane <= V) return rms_norm_reg_kernel<T, V><<<persistent, 256, 0, s>>>(x, w, out, rows, n, eps);
  TOKMIX_RMS_CASE(1)
  TOKMIX_RMS_CASE(2)
  TOKMIX_RMS_CASE(4)
  TOKMIX_RMS_CASE(8)
  TOKMIX_RMS_CASE(12)
  TOKMIX_RMS_CASE(16)
  TOKMIX_RMS_CASE(20)
  TOKMIX_RMS_CASE(24)
  TOKMIX_RMS_CASE(32)
#undef TOKMIX_RMS_CASE
  rms_norm_kernel<T><<<blocks, 256, 0, s>>>(x, w, out, rows, n, eps);
}

// ---------------------------------------------------------------------- SwiGLU + FP8 quantisation
// 16-lane maximum (xor offsets below 16 stay inside each half of the warp).
__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float abs_max8(uint4 v) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(__bfloat162float(e[j])));
  return a;
}

// amax times the fp32 reciprocal of 448: the rounding of the checker's division of a device tensor
// by a scalar, which torch evaluates as a multiplication by the scalar's reciprocal
__device__ __forceinline__ float block_scale(float amax, float eps) { return fmaxf(amax, eps) * (1.0f / 448.0f); }

// x * bf16(1/scale) rounded to bf16, then to e4m3 (round to nearest, saturating), 8 values -> 8
// bytes; two values per instruction (element 2j in the low byte of pair j)
__device__ __forceinline__ uint2 quant8(uint4 v, float scale) {
  const __nv_bfloat162 inv2 = __bfloat162bfloat162(__float2bfloat16_rn(__frcp_rn(scale)));  // 1 / scale rounded once
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t q[2] = {0u, 0u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 prod = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]), inv2);
    const uint32_t q2 = __nv_cvt_float2_to_fp8x2(__bfloat1622float2(prod), __NV_SATFINITE, __NV_E4M3);
    q[j >> 1] |= q2 << (16 * (j & 1));
  }
  return make_uint2(q[0], q[1]);
}

// Grid (m, ceil(n / 128 / 8)) of 128-thread CTAs: CTA (row, y) holds 8 half-warps, half-warp i
// takes block b = 8 y + i of the row (no integer division anywhere).
__global__ void __launch_bounds__(128) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                           __nv_bfloat16* __restrict__ out, uint8_t* __restrict__ xq,
                                                           float* __restrict__ xscale, int m, int n, float eps) {
  const int nb = n / 128;  // 128-column blocks per half of a row
  const int row = blockIdx.x;
  const int b = blockIdx.y * 8 + (threadIdx.x >> 4);
  const int sub = threadIdx.x & 15;
  const bool act = b < nb;
  const int col = b * 128 + 8 * sub;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * 2 * n;
  uint4 a = make_uint4(0u, 0u, 0u, 0u), c = a;
  if (act) {
    a = __ldcs(reinterpret_cast<const uint4*>(xr + col));      // x0 (also block b of x)
    c = __ldcs(reinterpret_cast<const uint4*>(xr + n + col));  // x1 (block nb + b of x)
  }
  // every lane reaches the shuffles, active or not
  const float amax_a = half_warp_max(abs_max8(a));
  const float amax_c = half_warp_max(abs_max8(c));
  if (!act) return;
  const float sa = block_scale(amax_a, eps), sc = block_scale(amax_c, eps);
  uint8_t* qr = xq + static_cast<size_t>(row) * 2 * n;
  __stcs(reinterpret_cast<uint2*>(qr + col), quant8(a, sa));
  __stcs(reinterpret_cast<uint2*>(qr + n + col), quant8(c, sc));
  if (sub == 0) {
    xscale[static_cast<size_t>(b) * m + row] = sa;
    xscale[static_cast<size_t>(nb + b) * m + row] = sc;
  }
  const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&a);
  const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&c);
  uint4 o;
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // x0 * (x1 * sigmoid(x1)), each product rounded to fp32 as the checker's
    const float x1 = __bfloat162float(e1[j]);
    // 1 / (1 + e^-x1) by the fast approximate divide: the correctly rounded reciprocal made the
    // outputs bit-identical to the checker's but cost 17 % of the kernel's time; with this one an
    // output differs from the checker's by at most one bf16 ulp (208 of 29.4M at M4096 N7168)
    const float sig = __fdividef(1.0f, 1.0f + expf(-x1));
    oe[j] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(e0[j]), __fmul_rn(x1, sig)));
  }
  __stcs(reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * n + col), o);
}

// -------------------------------------------------------------------------- partial rotary QKV
// out0 = x0 c - x1 s and out1 = x0 s + x1 c, every product and sum rounded separately
__device__ __forceinline__ float rot_lo(float x0, float x1, float c, float s) {
  return __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
}
__device__ __forceinline__ float rot_hi(float x0, float x1, float c, float s) {
  return __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

constexpr int kRopeHeadsPerWarp = 4;

// One warp per (token row, group of 4 heads); lane l < head_dim/8 owns vector l of each head.
// Requires head_dim <= 256 and a rope half that is a whole number of vectors.
__global__ void __launch_bounds__(256) qkv_rope_warp_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                            const float* __restrict__ cosv,
                                                            const float* __restrict__ sinv,
                                                            __nv_bfloat16* __restrict__ out, long long rows, int seq,
                                                            int heads, int head_dim, int nope, int rot_heads,
                                                            float sin_sign) {
  const int groups = (heads + kRopeHeadsPerWarp - 1) / kRopeHeadsPerWarp;
  const long long item = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= rows * groups) return;  // warp-uniform
  const long long row = item / groups;
  const int h0 = static_cast<int>(item - row * groups) * kRopeHeadsPerWarp;
  const int lane = threadIdx.x & 31;
  const int dvec = head_dim / 8, nope_vec = nope / 8, hvec = (head_dim - nope) / 16;
  const int half = (head_dim - nope) / 2;
  const size_t base = static_cast<size_t>(row) * heads * head_dim;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + base);
  uint4* dst = reinterpret_cast<uint4*>(out + base);
  const bool own = lane < dvec;
  uint4 v[kRopeHeadsPerWarp];
#pragma unroll
  for (int k = 0; k < kRopeHeadsPerWarp; ++k)
    v[k] = (own && h0 + k < heads) ? __ldcs(src + static_cast<size_t>(h0 + k) * dvec + lane)
                                   : make_uint4(0u, 0u, 0u, 0u);
  const int p = lane - nope_vec;  // vector index inside the rope columns
  const bool rope_lane = own && p >= 0;
  const bool first = p < hvec;  // first half of the pair (x0) or second (x1)
  const int partner = rope_lane ? (first ? lane + hvec : lane - hvec) : lane;
  float cs[8], sn[8];
  if (rope_lane && h0 < rot_heads) {
    const size_t t = static_cast<size_t>(row % seq) * half + static_cast<size_t>(first ? p : p - hvec) * 8;
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(cosv + t));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(cosv + t + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sinv + t));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(sinv + t + 4));
    cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
    sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
#pragma unroll
    for (int j = 0; j < 8; ++j) sn[j] *= sin_sign;
  }
#pragma unroll
  for (int k = 0; k < kRopeHeadsPerWarp; ++k) {
    uint4 pv;  // every lane shuffles: the partner vector of rope lanes, its own otherwise
    pv.x = __shfl_sync(0xffffffffu, v[k].x, partner);
    pv.y = __shfl_sync(0xffffffffu, v[k].y, partner);
    pv.z = __shfl_sync(0xffffffffu, v[k].z, partner);
    pv.w = __shfl_sync(0xffffffffu, v[k].w, partner);
    const int h = h0 + k;
    if (!own || h >= heads) continue;
    uint4 o = v[k];
    if (rope_lane && h < rot_heads) {
      const __nv_bfloat16* me = reinterpret_cast<const __nv_bfloat16*>(&v[k]);
      const __nv_bfloat16* pe = reinterpret_cast<const __nv_bfloat16*>(&pv);
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = __bfloat162float(me[j]), b = __bfloat162float(pe[j]);
        oe[j] = __float2bfloat16_rn(first ? rot_lo(a, b, cs[j], sn[j]) : rot_hi(b, a, cs[j], sn[j]));
      }
    }
    __stcs(dst + static_cast<size_t>(h) * dvec + lane, o);
  }
}

// Any other shape: one CTA per token row; vectors of untouched columns copied, pairs rotated one
// element at a time.
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
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const int h = i / dvec, c = i - h * dvec;
    if (h >= rot_heads || c < nope_vec) dst[i] = src[i];
  }
  for (int i = threadIdx.x; i < rot_heads * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    const size_t o0 = base + static_cast<size_t>(h) * head_dim + nope + j;
    const float x0 = __bfloat162float(qkv[o0]);
    const float x1 = __bfloat162float(qkv[o0 + half]);
    const float c = cosv[static_cast<size_t>(s) * half + j];
    const float sn = sin_sign * sinv[static_cast<size_t>(s) * half + j];
    out[o0] = __float2bfloat16_rn(rot_lo(x0, x1, c, sn));
    out[o0 + half] = __float2bfloat16_rn(rot_hi(x0, x1, c, sn));
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
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(TOKMIX_ERR_DEVICE, "tokmix_rms_norm: cannot query the SM count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TOKMIX_DTYPE_BF16)
    launch_rms_norm(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
                    static_cast<__nv_bfloat16*>(out), rows, n, eps, sms, s);
  else
    launch_rms_norm(static_cast<const __half*>(x), static_cast<const __half*>(weight), static_cast<__half*>(out), rows,
                    n, eps, sms, s);
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
  const int nb = n / 128;
  if ((nb + 7) / 8 > 65535) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_swiglu_input_quant: rows too long");
  if (const int rc = check_device()) return rc;
  const dim3 grid(static_cast<unsigned>(m), static_cast<unsigned>((nb + 7) / 8));
  swiglu_quant_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), static_cast<uint8_t*>(x_fp8), x_scale,
      m, n, eps);
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
  const int rot_heads = q_heads + kv_heads;
  const float sign = negative_sin ? -1.0f : 1.0f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rope_dim = head_dim - nope_dim;
  if (head_dim <= 256 && rope_dim % 16 == 0 && (rope_dim == 0 || (aligned16(cos) && aligned16(sin)))) {
    const long long warps = rows * ((heads + kRopeHeadsPerWarp - 1) / kRopeHeadsPerWarp);
    if ((warps + 7) / 8 > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_qkv_part_rope: too many rows");
    if (const int rc = check_device()) return rc;
    qkv_rope_warp_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(qkv), cos, sin, static_cast<__nv_bfloat16*>(out), rows, seq, heads, head_dim,
        nope_dim, rot_heads, sign);
  } else {
    if (rows > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_qkv_part_rope: too many rows");
    if (const int rc = check_device()) return rc;
    qkv_part_rope_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(qkv), cos, sin,
                                                                     static_cast<__nv_bfloat16*>(out), seq, heads,
                                                                     head_dim, nope_dim, rot_heads, sign);
  }
  return check_launch("tokmix_qkv_part_rope");
}
