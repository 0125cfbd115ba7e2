// gdn_decode.cu -- one decode step of the gated delta rule: one new token per sequence and value
// head, the fp32 state read once and written once (in place, or into a separate output state).
//
// Maths, per (sequence b, value head h, value row c) -- the reference's fp32 recurrence
// (kernels/qwen35moe_gdn_prefill.cu:55-99) for a single token, which its optimised prefill also
// special-cases (kernels_optimized/qwen35moe_gdn_prefill.cu:865-934, chunks with one token):
//   gamma = exp(g[b,h]);  kv = sum_i S[c][i] k[i];  delta = (v[c] - gamma kv) beta[b,h]
//   S[c][i] = gamma S[c][i] + k[i] delta;  o[c] = scale sum_i S[c][i] q[i]   (the updated S)
// with k, q of key head h % Hk.  State layout [b][h][c (value)][i (key)], fp32.
//
// Work per (b, h): 64 KB of state read and 64 KB written, ~1 KB of q/k/v/o -- HBM-bound, no
// tensor-core shape in it (two matrix-vector products and a rank-1 update per head).  One warp
// per value row: lane l holds S[c][4l .. 4l+3], so the warp moves the row's 512 bytes in one
// coalesced float4 access; both dot products are warp butterflies.  A CTA of 8 warps takes 32
// rows (4 per warp, their loads issued together so 2 KB per warp are in flight); 4 CTAs cover
// one (b, h).  No shared memory, no waits: nothing can hang.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "host_common.h"

namespace tokmix {
namespace gdn_decode {

constexpr int kD = 128;
constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 4;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;  // 32
constexpr int kCtasPerHead = kD / kRowsPerCta;      // 4

struct Params {
  const __nv_bfloat16* q;  // [batch, heads_k, 128]
  const __nv_bfloat16* k;  // [batch, heads_k, 128]
  const __nv_bfloat16* v;  // [batch, heads_v, 128]
  const float* g;          // [batch, heads_v]
  const float* beta;       // [batch, heads_v]
  const float* state_in;   // [batch, heads_v, 128, 128] or null (zero state); may equal state_out
  float* state_out;        // [batch, heads_v, 128, 128]
  __nv_bfloat16* out;      // [batch, heads_v, 128]
  int hk, hv;
  float scale;
};

__device__ __forceinline__ void unpack4(uint2 w, float (&f)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

__global__ void __launch_bounds__(kWarps * 32) gdn_decode_kernel(const Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x / kCtasPerHead;  // b * hv + h
  const int part = blockIdx.x - unit * kCtasPerHead;
  const int b = unit / p.hv, h = unit - b * p.hv;
  const int kh = h % p.hk;
  const int row0 = part * kRowsPerCta + warp * kRowsPerWarp;
  const size_t srow0 = (static_cast<size_t>(unit) * kD + row0) * kD;

  // the warp's rows first: the state is the only large read
  float4 s[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
    s[r] = p.state_in ? __ldcs(reinterpret_cast<const float4*>(p.state_in + srow0 + r * kD) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
  float kf[4], qf[4];
  unpack4(*(reinterpret_cast<const uint2*>(p.k + (static_cast<size_t>(b) * p.hk + kh) * kD) + lane), kf);
  unpack4(*(reinterpret_cast<const uint2*>(p.q + (static_cast<size_t>(b) * p.hk + kh) * kD) + lane), qf);
  const float gam = expf(p.g[unit]);
  const float bet = p.beta[unit];
  const __nv_bfloat16* vrow = p.v + static_cast<size_t>(unit) * kD + row0;

  float o[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float kv = warp_sum(s[r].x * kf[0] + s[r].y * kf[1] + s[r].z * kf[2] + s[r].w * kf[3]);
    const float delta = (__bfloat162float(vrow[r]) - gam * kv) * bet;
    s[r].x = gam * s[r].x + kf[0] * delta;
    s[r].y = gam * s[r].y + kf[1] * delta;
    s[r].z = gam * s[r].z + kf[2] * delta;
    s[r].w = gam * s[r].w + kf[3] * delta;
    o[r] = p.scale * warp_sum(s[r].x * qf[0] + s[r].y * qf[1] + s[r].z * qf[2] + s[r].w * qf[3]);
    __stcs(reinterpret_cast<float4*>(p.state_out + srow0 + r * kD) + lane, s[r]);
  }
  if (lane == 0) {  // the warp's 4 consecutive outputs: one 8-byte store
    const __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]);
    const __nv_bfloat162 o23 = __floats2bfloat162_rn(o[2], o[3]);
    uint2 w;
    w.x = *reinterpret_cast<const uint32_t*>(&o01);
    w.y = *reinterpret_cast<const uint32_t*>(&o23);
    *reinterpret_cast<uint2*>(p.out + static_cast<size_t>(unit) * kD + row0) = w;
  }
}

}  // namespace gdn_decode
}  // namespace tokmix

extern "C" int tokmix_gdn_decode(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                 const float* state_in, float* state_out, void* out, int batch, int heads_k,
                                 int heads_v, int head_dim_k, int head_dim_v, float scale, int io_dtype,
                                 void* stream) {
  using namespace tokmix;
  using namespace tokmix::gdn_decode;
  if (batch < 0 || heads_k <= 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_decode: negative batch or non-positive head count");
  if (heads_v % heads_k != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_decode: heads_v (%d) must be a multiple of heads_k (%d)",
                heads_v, heads_k);
  if (head_dim_k != kD || head_dim_v != kD)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_decode: head dims must be 128 (got %d, %d)", head_dim_k,
                head_dim_v);
  if (io_dtype != TOKMIX_DTYPE_BF16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_decode: only bf16 q/k/v/out are supported by the kernel");
  if (!std::isfinite(scale)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_decode: scale must be finite");
  if (batch == 0) return TOKMIX_OK;
  if (!q || !k || !v || !g || !beta || !state_out || !out)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_decode: null pointer argument");
  for (const void* ptr : {q, k, v, static_cast<const void*>(state_in), static_cast<const void*>(state_out),
                          static_cast<const void*>(out)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_decode: tensors must be 16-byte aligned");
  const long long ctas = static_cast<long long>(batch) * heads_v * kCtasPerHead;
  if (ctas > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_decode: problem too large");
  if (const int rc = check_device()) return rc;
  Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.g = g;
  p.beta = beta;
  p.state_in = state_in;
  p.state_out = state_out;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.hk = heads_k;
  p.hv = heads_v;
  p.scale = scale;
  gdn_decode_kernel<<<static_cast<unsigned>(ctas), kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("tokmix_gdn_decode");
}
