// gdn_common.cuh -- building blocks shared by the GDN prefill kernels (gdn_prefill.cu: one CTA per
// (sequence, value head) doing everything; gdn_split.cu: a chunk-parallel preparation kernel and
// a state-chain kernel).  Chunk = 64 tokens; head dims 128.  See gdn_prefill.cu for the maths.
#pragma once

#include <cuda_bf16.h>

#include "sm100.cuh"

namespace tokmix {
namespace gdn {

constexpr int kC = 64;    // tokens per chunk
constexpr int kD = 128;   // head dim (keys and values)
constexpr int kLds = 68;  // fp32 row stride of the solve matrices L and X (64 + 4: conflict-free rows)

// Where a chunk's gates come from: g and beta as given, or -- when `a` is not null -- the
// Qwen3.5 gated-delta-net gates computed from the raw projections a, b [tokens, heads_v] (bf16
// or fp32) and the per-head A_log, dt_bias, with the same arithmetic as the separate gates pass
// (gdn_preprocess.cu), so both routes give the same bits:
//   g = -exp(A_log[h]) softplus(a + dt_bias[h]),   beta = sigmoid(b)
struct GateSource {
  const void* a;
  const void* b;
  const float* a_log;
  const float* dt_bias;
  int bf16;  // a, b are bf16 (else fp32)
};

// softplus(x) = log(1 + e^x); for x > 20, e^x exceeds 4e8 and log(1 + e^x) equals x in fp32
__device__ __forceinline__ float gate_softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// g and beta of element idx (= token * heads_v + h)
__device__ __forceinline__ void load_gates(const float* g, const float* beta, const GateSource& gs, size_t idx, int h,
                                           float& gv, float& bv) {
  if (gs.a == nullptr) {
    gv = g[idx];
    bv = beta[idx];
    return;
  }
  const float a = gs.bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(gs.a)[idx])
                          : static_cast<const float*>(gs.a)[idx];
  const float b = gs.bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(gs.b)[idx])
                          : static_cast<const float*>(gs.b)[idx];
  gv = -expf(gs.a_log[h]) * gate_softplus(a + gs.dt_bias[h]);
  bv = 1.0f / (1.0f + expf(-b));
}

// Sum of squares of four values in a fixed order (explicitly rounded, so every caller gets the
// same bits): the per-lane step of the row L2 normalisation (qk_l2norm).
__device__ __forceinline__ float sumsq4(float a, float b, float c, float d) {
  return __fmaf_rn(d, d, __fmaf_rn(c, c, __fmaf_rn(b, b, __fmul_rn(a, a))));
}

// x / sqrt(sum x^2 + eps) of one bf16 row of 128 held in shared memory as the 128-byte rows of two
// 128-byte-swizzled 64-column boxes (half0: elements 0-63, half1: 64-127; swizzle phase r7 = the
// row's index & 7), in place.  The sum is formed exactly as the normalisation pass over global
// memory forms it (gdn_preprocess.cu: 32 lanes take 4 consecutive elements each, then an XOR
// butterfly over offsets 16 .. 1), so both give the same bits.  Returns the scaling factor.
__device__ __forceinline__ float l2norm_row_sw128(uint8_t* half0, uint8_t* half1, int r7, float eps) {
  float part[32];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint8_t* base = h ? half1 : half0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // 16-byte chunk j holds elements 64h + 8j .. +7
      const uint4 w = *reinterpret_cast<const uint4*>(base + ((j ^ r7) << 4));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.z));
      const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.w));
      part[16 * h + 2 * j] = sumsq4(a.x, a.y, b.x, b.y);
      part[16 * h + 2 * j + 1] = sumsq4(c.x, c.y, d.x, d.y);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    float nxt[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) nxt[l] = __fadd_rn(part[l], part[l ^ off]);
#pragma unroll
    for (int l = 0; l < 32; ++l) part[l] = nxt[l];
  }
  const float inv = rsqrtf(part[0] + eps);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint8_t* base = h ? half1 : half0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 w = *reinterpret_cast<const uint4*>(base + ((j ^ r7) << 4));
      uint32_t* e = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&e[q]));
        e[q] = pack_bf16x2(f.x * inv, f.y * inv);
      }
      *reinterpret_cast<uint4*>(base + ((j ^ r7) << 4)) = w;
    }
  }
  return inv;
}

// The normalised row (as above) copied to global memory in plain order: 128 bf16, 16-byte aligned.
__device__ __forceinline__ void copy_row_sw128(const uint8_t* half0, const uint8_t* half1, int r7, __nv_bfloat16* dst) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint8_t* base = h ? half1 : half0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      reinterpret_cast<uint4*>(dst)[8 * h + j] = *reinterpret_cast<const uint4*>(base + ((j ^ r7) << 4));
  }
}

struct ChunkParams {
  float beta[kC];  // write strength (0 for tokens past the sequence end)
  float g2[kC];    // in-chunk inclusive prefix sum of g, in log2 units
  float eg[kC];    // exp(G_t) (0 past the end)
  float egr[kC];   // exp(G_C - G_t) (0 past the end)
  float gamma_c;   // exp(G_C)
  int n_valid;
  int pad[62];
};
constexpr int kParamsBytes = 1280;
static_assert(sizeof(ChunkParams) == kParamsBytes, "params slot size");

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// write 32 bf16 values (16 packed uint32) as half `h` (bytes [64h, 64h+64)) of row `row` of a
// 128-byte-swizzled tile
__device__ __forceinline__ void store_half_row_sw128(uint8_t* tile, int row, int h, const uint32_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int chunk = 4 * h + j;
    *reinterpret_cast<uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4)) =
        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int row, const uint32_t (&v)[32]) {
  store_half_row_sw128(tile, row, 0, *reinterpret_cast<const uint32_t(*)[16]>(&v[0]));
  store_half_row_sw128(tile, row, 1, *reinterpret_cast<const uint32_t(*)[16]>(&v[16]));
}

// x = hi + lo as two bf16 operands: hi = x truncated to bf16 (its top 16 bits, exact), lo =
// the exact fp32 remainder rounded to bf16.  |x - hi - lo| <= 2^-16 |x|.
__device__ __forceinline__ uint32_t hi_pack(float x0, float x1) {
  return __byte_perm(__float_as_uint(x0), __float_as_uint(x1), 0x7632);
}
__device__ __forceinline__ uint32_t lo_pack(float x0, float x1) {
  return pack_bf16x2(x0 - __uint_as_float(__float_as_uint(x0) & 0xFFFF0000u),
                     x1 - __uint_as_float(__float_as_uint(x1) & 0xFFFF0000u));
}
__device__ __forceinline__ void split_pack(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = hi_pack(x0, x1);
  lo = lo_pack(x0, x1);
}

// 32 fp32 values x[OFF, OFF+32) (raw bits) -> hi and lo bf16 copies, 16 TMEM columns each
template <int OFF>
__device__ __forceinline__ void store_split32(uint32_t hi_addr, uint32_t lo_addr, const uint32_t (&x)[64]) {
  uint32_t hi[16], lo[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    split_pack(__uint_as_float(x[OFF + 2 * j]), __uint_as_float(x[OFF + 2 * j + 1]), hi[j], lo[j]);
  tmem_st16(hi_addr, hi);
  tmem_st16(lo_addr, lo);
}

// K-major tile of two 64-column boxes `box_bytes` apart: descriptor of the 16-element k step kk
__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int kk, uint32_t box_bytes) {
  return make_sdesc_sw128(base + (kk >> 2) * box_bytes + (kk & 3) * 32, 16, 1024);
}

// Decay prefix sums of one chunk (one warp; lane l holds tokens 2l, 2l+1): g and beta of the
// chunk's tokens (0 past the end) -> ChunkParams.
__device__ __forceinline__ void chunk_decay_params(ChunkParams& pc, float ga, float gb, float ba, float bb,
                                                   int n_valid, int lane) {
  const int t0 = 2 * lane, t1 = 2 * lane + 1;
  float incl = ga + gb;  // inclusive scan of pair sums
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  const float G0 = incl - gb;
  const float G1 = incl;
  const float GC = __shfl_sync(0xffffffffu, incl, 31);
  constexpr float kLog2e = 1.4426950408889634f;
  pc.beta[t0] = ba;
  pc.beta[t1] = bb;
  pc.g2[t0] = G0 * kLog2e;
  pc.g2[t1] = G1 * kLog2e;
  pc.eg[t0] = t0 < n_valid ? expf(G0) : 0.0f;
  pc.eg[t1] = t1 < n_valid ? expf(G1) : 0.0f;
  pc.egr[t0] = t0 < n_valid ? expf(GC - G0) : 0.0f;
  pc.egr[t1] = t1 < n_valid ? expf(GC - G1) : 0.0f;
  if (lane == 0) {
    pc.gamma_c = expf(GC);
    pc.n_valid = n_valid;
  }
}

// Row t of L = beta_t exp(G_t - G_s) (k_t . k_s), s < t, from row t of K K^T -> Ls[t][*]
__device__ __forceinline__ void l_row(const uint32_t (&row)[64], const ChunkParams& pc, int t, float* Ls) {
  const float gt = pc.g2[t];
  const float bt = pc.beta[t];
  float* lrow = Ls + t * kLds;
#pragma unroll
  for (int s4 = 0; s4 < 64; s4 += 4) {
    const float4 g4 = *reinterpret_cast<const float4*>(&pc.g2[s4]);
    float4 val;
    val.x = s4 + 0 < t ? bt * ex2_approx(gt - g4.x) * __uint_as_float(row[s4 + 0]) : 0.0f;
    val.y = s4 + 1 < t ? bt * ex2_approx(gt - g4.y) * __uint_as_float(row[s4 + 1]) : 0.0f;
    val.z = s4 + 2 < t ? bt * ex2_approx(gt - g4.z) * __uint_as_float(row[s4 + 2]) : 0.0f;
    val.w = s4 + 3 < t ? bt * ex2_approx(gt - g4.w) * __uint_as_float(row[s4 + 3]) : 0.0f;
    *reinterpret_cast<float4*>(lrow + s4) = val;
  }
}

// Row t of P = scale exp(G_t - G_s) (q_t . k_s), s <= t, from row t of Q K^T, as 32 packed bf16
// pairs (p_row below stores it)
__device__ __forceinline__ void p_row_pack(const uint32_t (&row)[64], const ChunkParams& pc, int t, float scale,
                                           uint32_t (&prow)[32]) {
  const float gt = pc.g2[t];
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const int s0 = 2 * j;
    const float4 g4 = *reinterpret_cast<const float4*>(&pc.g2[s0]);
    const float p0 = s0 + 0 <= t ? __uint_as_float(row[s0 + 0]) * ex2_approx(gt - g4.x) * scale : 0.0f;
    const float p1 = s0 + 1 <= t ? __uint_as_float(row[s0 + 1]) * ex2_approx(gt - g4.y) * scale : 0.0f;
    const float p2 = s0 + 2 <= t ? __uint_as_float(row[s0 + 2]) * ex2_approx(gt - g4.z) * scale : 0.0f;
    const float p3 = s0 + 3 <= t ? __uint_as_float(row[s0 + 3]) * ex2_approx(gt - g4.w) * scale : 0.0f;
    prow[j] = pack_bf16x2(p0, p1);
    prow[j + 1] = pack_bf16x2(p2, p3);
  }
}

// Row t of P (above) -> the P tile ([t][s] bf16, 128-byte swizzle)
__device__ __forceinline__ void p_row(const uint32_t (&row)[64], const ChunkParams& pc, int t, float scale,
                                      uint8_t* p_tile) {
  uint32_t prow[32];
  p_row_pack(row, pc, t, scale, prow);
  store_row_sw128(p_tile, t, prow);
}

// Scales row t (128 bf16 in two 64-column boxes `box_bytes` apart, swizzled rows of 128 B) by f,
// in place.  The whole row is rewritten, so the swizzle does not matter.
__device__ __forceinline__ void scale_row_inplace(uint8_t* box0_row, int box_bytes, float f) {
#pragma unroll
  for (int bx = 0; bx < 2; ++bx) {
    uint4 q8[8];
    uint8_t* rowp = box0_row + bx * box_bytes;
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[j] = *reinterpret_cast<const uint4*>(rowp + (j << 4));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&q8[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 b2 = *reinterpret_cast<__nv_bfloat162*>(&w[e]);
        const float2 fl = __bfloat1622float2(b2);
        w[e] = pack_bf16x2(fl.x * f, fl.y * f);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(rowp + (j << 4)) = q8[j];
  }
}

// Scales row t (128 bf16 in two 64-column boxes, swizzled rows of 128 B) by f and writes it to
// the same row of another pair of boxes (possibly in global memory); both row addresses have
// the same (row & 7), so the 16-byte chunks keep their swizzled positions.
__device__ __forceinline__ void scale_row_copy(const uint8_t* src_box0_row, int src_box_bytes, uint8_t* dst_box0_row,
                                               int dst_box_bytes, float f) {
#pragma unroll
  for (int bx = 0; bx < 2; ++bx) {
    uint4 q8[8];
    const uint8_t* srow = src_box0_row + bx * src_box_bytes;
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[j] = *reinterpret_cast<const uint4*>(srow + (j << 4));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&q8[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 b2 = *reinterpret_cast<__nv_bfloat162*>(&w[e]);
        const float2 fl = __bfloat1622float2(b2);
        w[e] = pack_bf16x2(fl.x * f, fl.y * f);
      }
    }
    uint8_t* drow = dst_box0_row + bx * dst_box_bytes;
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(drow + (j << 4)) = q8[j];
  }
}

// Row layout of the 64x64 fp32 matrix X of the solve (a template parameter of the functions that
// use it).  at(r, c) is the address of X[r][c]; for c a multiple of 4, X[r][c..c+3] are contiguous
// and 16-byte aligned.
struct PaddedRows {  // rows of kLds floats
  float* p;
  __device__ __forceinline__ float* at(int r, int c) const { return p + r * kLds + c; }
};

struct NoSideWork {
  __device__ __forceinline__ void operator()(int) const {}
};

// X = (I + L)^-1 (unit lower triangular, fp32), 128 threads meeting at named barrier `bar`, by
// recursive doubling over 16x16 blocks: the four diagonal blocks D_b by forward substitution
// (one column per thread of threads [d_lo, d_lo + 64); the other 64 threads run side(tid)
// meanwhile, which must not touch L or X); the two 32x32 diagonal blocks E_0,
// E_1 from X[2p+1, 2p] = -D_{2p+1} L[2p+1, 2p] D_{2p}; the lower 32x32 block as -E_1 L[1, 0] E_0.
// Products are staged in X's strictly upper blocks, which nothing else reads; the diagonal
// blocks hold explicit zeros above their diagonal.  Ends with a barrier: X is complete.
template <class XM, class Side = NoSideWork>
__device__ __forceinline__ void solve_inverse(const float* Ls, XM X, int tid, int bar, int d_lo = 64,
                                              Side side = Side{}) {
  if (tid >= d_lo && tid < d_lo + 64) {
    const int b = (tid - d_lo) >> 4, j = tid & 15;
    const float* lb16 = Ls + 16 * b * kLds + 16 * b;
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = (i == j) ? 1.0f : 0.0f;
#pragma unroll
    for (int s = 0; s < 15; ++s) {
      const float xs = acc[s];
#pragma unroll
      for (int i = s + 1; i < 16; ++i) acc[i] = fmaf(-lb16[i * kLds + s], xs, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) *X.at(16 * b + i, 16 * b + j) = acc[i];
  } else {
    side(tid);
  }
  named_sync(bar, 128);
  {  // pairs p: X[R + rr][C + c4..c4+3], R = 16(2p+1), C = 32p
    const int pr = tid >> 6, q = tid & 63, rr = q >> 2, c4 = (q & 3) * 4;
    const int R = 16 * (2 * pr + 1), C = 32 * pr;
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 16; ++k) {  // Y = L[R.., C..] D_{2p}
      const float l = Ls[(R + rr) * kLds + C + k];
      const float4 d = *reinterpret_cast<const float4*>(X.at(C + k, C + c4));
      y.x = fmaf(l, d.x, y.x);
      y.y = fmaf(l, d.y, y.y);
      y.z = fmaf(l, d.z, y.z);
      y.w = fmaf(l, d.w, y.w);
    }
    *reinterpret_cast<float4*>(X.at(C + rr, R + c4)) = y;  // staged in block (2p, 2p+1)
    named_sync(bar, 128);
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) {  // X[R.., C..] = -D_{2p+1} Y
      const float dm = *X.at(R + rr, R + m);
      const float4 ym = *reinterpret_cast<const float4*>(X.at(C + m, R + c4));
      z.x = fmaf(dm, ym.x, z.x);
      z.y = fmaf(dm, ym.y, z.y);
      z.z = fmaf(dm, ym.z, z.z);
      z.w = fmaf(dm, ym.w, z.w);
    }
    *reinterpret_cast<float4*>(X.at(R + rr, C + c4)) = make_float4(-z.x, -z.y, -z.z, -z.w);
  }
  named_sync(bar, 128);
  {  // lower 32x32 block.  Thread: row r of 32, columns 4q..4q+3 and 16+4q..16+4q+3.
    const int r = tid >> 2, q4 = (tid & 3) * 4;
    float4 ya = make_float4(0.f, 0.f, 0.f, 0.f), yb = ya;
    const float* lrow = Ls + (32 + r) * kLds;
#pragma unroll
    for (int k = 0; k < 32; ++k) {  // Y = L[32.., 0..32] E_0   (E_0 block (0,1) is not read)
      const float l = lrow[k];
      const float4 xa = *reinterpret_cast<const float4*>(X.at(k, q4));
      ya.x = fmaf(l, xa.x, ya.x);
      ya.y = fmaf(l, xa.y, ya.y);
      ya.z = fmaf(l, xa.z, ya.z);
      ya.w = fmaf(l, xa.w, ya.w);
      if (k >= 16) {
        const float4 xb = *reinterpret_cast<const float4*>(X.at(k, 16 + q4));
        yb.x = fmaf(l, xb.x, yb.x);
        yb.y = fmaf(l, xb.y, yb.y);
        yb.z = fmaf(l, xb.z, yb.z);
        yb.w = fmaf(l, xb.w, yb.w);
      }
    }
    *reinterpret_cast<float4*>(X.at(r, 32 + q4)) = ya;  // staged in rows 0-31, cols 32-63
    *reinterpret_cast<float4*>(X.at(r, 48 + q4)) = yb;
    named_sync(bar, 128);
    float4 za = make_float4(0.f, 0.f, 0.f, 0.f), zb = za;
#pragma unroll
    for (int m = 0; m < 16; ++m) {  // X[32.., 0..32] = -E_1 Y   (rows 32-47: D_2 only)
      const float e = *X.at(32 + r, 32 + m);
      const float4 a = *reinterpret_cast<const float4*>(X.at(m, 32 + q4));
      const float4 b = *reinterpret_cast<const float4*>(X.at(m, 48 + q4));
      za.x = fmaf(e, a.x, za.x);
      za.y = fmaf(e, a.y, za.y);
      za.z = fmaf(e, a.z, za.z);
      za.w = fmaf(e, a.w, za.w);
      zb.x = fmaf(e, b.x, zb.x);
      zb.y = fmaf(e, b.y, zb.y);
      zb.z = fmaf(e, b.z, zb.z);
      zb.w = fmaf(e, b.w, zb.w);
    }
    if (r >= 16) {  // warp-uniform: rows 48-63 also take X[3, 2] and D_3
#pragma unroll
      for (int m = 16; m < 32; ++m) {
        const float e = *X.at(32 + r, 32 + m);
        const float4 a = *reinterpret_cast<const float4*>(X.at(m, 32 + q4));
        const float4 b = *reinterpret_cast<const float4*>(X.at(m, 48 + q4));
        za.x = fmaf(e, a.x, za.x);
        za.y = fmaf(e, a.y, za.y);
        za.z = fmaf(e, a.z, za.z);
        za.w = fmaf(e, a.w, za.w);
        zb.x = fmaf(e, b.x, zb.x);
        zb.y = fmaf(e, b.y, zb.y);
        zb.z = fmaf(e, b.z, zb.z);
        zb.w = fmaf(e, b.w, zb.w);
      }
    }
    *reinterpret_cast<float4*>(X.at(32 + r, q4)) = make_float4(-za.x, -za.y, -za.z, -za.w);
    *reinterpret_cast<float4*>(X.at(32 + r, 16 + q4)) = make_float4(-zb.x, -zb.y, -zb.z, -zb.w);
  }
  named_sync(bar, 128);
}

// T = X diag(beta) and TG = T diag(e^G) as MN-major ([s][t]) hi/lo bf16 tiles (hi at tile, lo at
// tile + lo_off; shared or global memory), 128 threads: thread = (row s, token half).  Entries
// above the diagonal are 0.
template <class XM>
__device__ __forceinline__ void write_t_tiles(XM X, const ChunkParams& pc, int tid, uint8_t* t_tile,
                                              uint8_t* tg_tile, int t_lo_off = 8192, int tg_lo_off = 8192) {
  const int s = tid & 63, half = tid >> 6;
  float xv[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int t = 32 * half + i;
    xv[i] = t >= s ? *X.at(t, s) : 0.0f;
  }
  const float w0 = pc.beta[s];
  const float w1 = w0 * pc.eg[s];
#pragma unroll
  for (int qq = 0; qq < 2; ++qq) {
    const float w = qq ? w1 : w0;
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) split_pack(xv[2 * i] * w, xv[2 * i + 1] * w, hi[i], lo[i]);
    uint8_t* tile = qq ? tg_tile : t_tile;
    store_half_row_sw128(tile, s, half, hi);
    store_half_row_sw128(tile + (qq ? tg_lo_off : t_lo_off), s, half, lo);
  }
}

// Row k of W^T (64 tokens, fp32 raw bits) -> row k of the -W hi/lo tiles ([k][t], hi at w_tile,
// lo at w_tile + lo_off)
__device__ __forceinline__ void w_row(const uint32_t (&row)[64], int k, uint8_t* w_tile, int lo_off = 16384) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      split_pack(-__uint_as_float(row[32 * half + 2 * j]), -__uint_as_float(row[32 * half + 2 * j + 1]), hi[j], lo[j]);
    store_half_row_sw128(w_tile, k, half, hi);
    store_half_row_sw128(w_tile + lo_off, k, half, lo);
  }
}

}  // namespace gdn
}  // namespace tokmix
