// gdn_prefill.cu -- chunked gated-delta-rule prefill for sm_100a (B200).
//
// Reference path replaced: kernels_optimized/qwen35moe_gdn_prefill.cu:683-1161 (precompute +
// chunk-scan kernels) behind qwen35moe_gdn_prefill_bf16tc (:1203-1264).  Maths: the fp32
// recurrence kernels/qwen35moe_gdn_prefill.cu:55-99 (value head h reads key head h % Hk,
// state layout [v][k], output computed with the updated state).
//
// Chunked form used here (C = 64 tokens, in-chunk cumulative log decay G_t, incoming state S0):
//   L_ts  = beta_t exp(G_t - G_s) (k_t . k_s)          s < t
//   T     = (I + L)^-1 diag(beta)                      (unit-lower inverse, fp32, blocked 16x16)
//   W     = T diag(e^G) K                              (tensor core; T diag(e^G) as bf16 hi + lo)
//   Delta = T V - W S0^T                               (tensor core; T as hi + lo; W S0^T as the
//                                                       3-term product W_hi S_hi + W_lo S_hi + W_hi S_lo)
//   O     = scale (diag(e^G) Q S0^T + P Delta),  P_ts = exp(G_t - G_s)(q_t . k_s), s <= t
//   S     = e^{G_C} S0 + (diag(e^{G_C - G}) Delta)^T K (tensor core; Delta' split hi + lo)
// Every contraction is an M=128 tcgen05 MMA because the CTA keeps the VALUE dimension on the
// 128 TMEM lanes ("transposed" products: Delta^T, O^T, S with lane = value row; W^T with
// lane = key row).  The fp32 master state never leaves TMEM between chunks; a hi + lo bf16 copy
// in shared memory is the MMA operand for the next chunk.  The hi/lo splits keep every product
// that feeds the state at ~16 significant bits, so the fp32 final state stays within 1e-3
// relative of the fp32 recurrence even when the decay is weak.
//
// One CTA processes one (sequence, value head) unit, all its chunks in order.  Warp roles:
//   warps 0-3   state chain: Delta pass (Delta -> bf16 operands in TMEM), state pass (S ->
//               bf16 shared copy, pre-scale by the next chunk's decay), initial/final state
//   warps 4-7   operands: decay prefix sums, QK/KK read-out (P tile, e^G-scaled Q, L rows),
//               W pass (W^T -> -W bf16 tile), output pass (O^T -> global)
//   warps 8-9   triangular solve -> T (hi/lo) and T diag(e^G) tiles
//   warp 10     TMA producer (stacked Q/K chunk tile, V chunk tile)
//   warp 11     TMEM owner and MMA issuer for the state-independent groups; it polls the
//               hand-off barriers and issues whichever group is ready.  The state-dependent
//               groups are issued by the warps that produce their inputs, so the state chain
//               never waits behind the next chunk's preparation.
// Hand-off barriers are two-slot arrays indexed by chunk parity.  All waits are bounded.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "host_common.h"
#include "sm100.cuh"

namespace tokmix {
namespace gdn {

constexpr int kC = 64;     // tokens per chunk
constexpr int kD = 128;    // head dim (keys and values)
constexpr int kThreads = 384;
constexpr int kWarpTma = 10;
constexpr int kWarpMma = 11;

// TMEM columns
constexpr uint32_t kColS = 0;      // state S[v][k] fp32, 128 cols
constexpr uint32_t kColX0 = 128;   // Delta^T fp32 (64 cols) then bf16 A operands (96 cols), 2 slots
constexpr uint32_t kColX1 = 224;
constexpr uint32_t kColO = 320;    // O^T fp32, 64 cols
constexpr uint32_t kColW = 384;    // W^T fp32 (lane = key row), 64 cols
constexpr uint32_t kColQK = 448;   // lanes 0-63: Q K^T, lanes 64-127: K K^T, 64 cols

// shared memory layout (bytes; every MMA tile starts on a 1024-byte boundary)
constexpr int kSlotBytes = 32768;                  // stacked [Q;K] chunk tile: 2 boxes of 128 rows x 128 B
constexpr int kOffSlot0 = 0;                       //   rows 0-63 of a box: Q (scaled in place to e^G Q)
constexpr int kOffSlot1 = kSlotBytes;              //   rows 64-127: K
constexpr int kOffV = 2 * kSlotBytes;              // V chunk tile: 2 boxes of 64 rows x 128 B
constexpr int kOffP = kOffV + 16384;               // P [t][s] bf16
constexpr int kOffThi = kOffP + 8192;              // T hi [t][s]
constexpr int kOffTlo = kOffThi + 8192;            // T lo
constexpr int kOffTGhi = kOffTlo + 8192;           // T diag(e^G) hi
constexpr int kOffTGlo = kOffTGhi + 8192;          // T diag(e^G) lo
constexpr int kOffWhi = kOffTGlo + 8192;           // -W hi as [k][t], 128 rows x 128 B
constexpr int kOffWlo = kOffWhi + 16384;           // -W lo
constexpr int kOffShi = kOffWlo + 16384;           // state copy hi [v][k]: 2 boxes of 128 rows x 128 B
constexpr int kOffSlo = kOffShi + 32768;           // state copy lo
constexpr int kOffParams = kOffSlo + 32768;
constexpr int kParamsBytes = 1280;
constexpr int kSmemBytes = kOffParams + 2 * kParamsBytes;
// The triangular solve reads L from fp32 scratch that aliases the T hi/lo tiles and keeps its
// solved columns in a buffer that aliases the T diag(e^G) tiles; it writes the tiles only after
// both have been read into registers.  L is stored column-major: scratch[s * 64 + t] = L[t][s].
constexpr int kOffScratch = kOffThi;
static_assert(kOffTGhi - kOffThi >= 64 * 64 * 4 && kOffWhi - kOffTGhi >= 64 * 64 * 4, "solve buffers");
static_assert(kSmemBytes + 1024 <= 227 * 1024, "shared memory budget");

struct ChunkParams {
  float beta[kC];         // write strength (0 for tokens past the sequence end)
  float g2[kC];           // in-chunk inclusive prefix sum of g, in log2 units
  float eg[kC];           // exp(G_t) (0 past the end)
  float egr[kC];          // exp(G_C - G_t) (0 past the end)
  float gamma_c;          // exp(G_C)
  int n_valid;
  int pad[62];
};
static_assert(sizeof(ChunkParams) == kParamsBytes, "params slot size");

struct Params {
  const float* g;
  const float* beta;
  const float* state_in;
  float* state_out;
  __nv_bfloat16* out;
  const int32_t* cu_seqlens;
  const int32_t* seq_order;
  int hk, hv;
  float scale;
  uint32_t* status;
};

// Hand-off barriers, each a 2-slot array indexed by chunk parity (event of chunk c lives in slot
// c & 1 and completes its (c >> 1)-th phase).  Every producer of chunk c+2's event causally
// follows every waiter of chunk c's event, so no waiter can fall two phases behind.
struct Barriers {
  uint64_t in_full[2], v_full[2], v_free[2];
  uint64_t qk_done[2], qk_read[2], g_ready[2], prep1[2];
  uint64_t w_done[2], wneg[2], delta[2], da_done[2];
  uint64_t snew[2], s_ready[2], o_done[2];
  uint64_t p_ready[2], t3b[2];
};

__device__ __forceinline__ bool wait_c(uint64_t* bars, int c, uint32_t* status, uint32_t code) {
  return mbar_wait(&bars[c & 1], (c >> 1) & 1, status, code);
}
__device__ __forceinline__ bool test_c(uint64_t* bars, int c) { return mbar_test(&bars[c & 1], (c >> 1) & 1); }
// Warp-uniform wait: tcgen05.ld/st are warp-collective, so a warp continues or stops as a whole.
__device__ __forceinline__ bool wait_c_warp(uint64_t* bars, int c, uint32_t* status, uint32_t code) {
  return __all_sync(0xffffffffu, wait_c(bars, c, status, code));
}

// Optional phase trace (build with -DTOKMIX_GDN_TRACE): %globaltimer stamps of CTA 0, indexed
// by event and chunk, read back with tokmix_gdn_trace_read().  Compiled out otherwise.
#ifdef TOKMIX_GDN_TRACE
constexpr int kTraceChunks = 64;
constexpr int kTraceEvents = 24;
__device__ unsigned long long g_trace[kTraceEvents * kTraceChunks];
#define GDN_TRACE(ev, c)                                                          \
  do {                                                                            \
    if (blockIdx.x == 0 && (c) < kTraceChunks) g_trace[(ev) * kTraceChunks + (c)] = global_timer_ns(); \
  } while (0)
#else
#define GDN_TRACE(ev, c) \
  do {                   \
  } while (0)
#endif

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
__device__ __forceinline__ void split_pack(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const uint32_t b0 = __float_as_uint(x0), b1 = __float_as_uint(x1);
  hi = __byte_perm(b0, b1, 0x7632);
  lo = pack_bf16x2(x0 - __uint_as_float(b0 & 0xFFFF0000u), x1 - __uint_as_float(b1 & 0xFFFF0000u));
}

// Writes 64 fp32 state values (columns [64*half, 64*half+64) of row v) as the hi and lo bf16
// state copies (box `half` of each).
__device__ __forceinline__ void store_state_half(uint8_t* smem, int v, int half, const uint32_t (&sv)[64]) {
#pragma unroll
  for (int q4 = 0; q4 < 2; ++q4) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      split_pack(__uint_as_float(sv[32 * q4 + 2 * j]), __uint_as_float(sv[32 * q4 + 2 * j + 1]), hi[j], lo[j]);
    store_half_row_sw128(smem + kOffShi + half * 16384, v, q4, hi);
    store_half_row_sw128(smem + kOffSlo + half * 16384, v, q4, lo);
  }
}

__device__ __forceinline__ void output_pass(const Params& p, uint32_t lane_base, int tok0, int len, int cp, int h,
                                            int r) {
  const int nv = min(kC, len - cp * kC);
  uint32_t row[64];
  tmem_ld64(lane_base + kColO, row);
  if (r == 0) GDN_TRACE(20, cp);
  __nv_bfloat16* dst = p.out + (static_cast<size_t>(tok0 + cp * kC) * p.hv + h) * kD + r;
  const size_t tstride = static_cast<size_t>(p.hv) * kD;
#pragma unroll
  for (int t = 0; t < kC; ++t)
    if (t < nv) dst[t * tstride] = __float2bfloat16_rn(__uint_as_float(row[t]) * p.scale);
}

// K-major tile of 2 boxes (16 KB apart): descriptor of the 16-element k step kk
__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}

// T3a  Delta^T += S_hi (-W_hi)^T + S_lo (-W_hi)^T + S_hi (-W_lo)^T   (M=128 v, N=64 t, K=128 k)
__device__ __forceinline__ void issue_t3a(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id_sw = make_idesc(128, 64, 1, 0, 1);  // A K-major (S), B MN-major (-W as [k][t])
  const uint32_t colx = (c & 1) ? kColX1 : kColX0;
#pragma unroll
  for (int term = 0; term < 3; ++term) {
    const uint32_t sa = smem_u32(smem + (term == 1 ? kOffSlo : kOffShi));
    const uint32_t wa = smem_u32(smem + (term == 2 ? kOffWlo : kOffWhi));
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16_ss(tbase + colx, kmaj_desc(sa, kk), make_sdesc_sw128(wa + kk * 2048, 16384, 1024), id_sw, 1u);
  }
}

// T3b  O^T = S_hi (e^G Q)^T   (M=128 v, N=64 t, K=128 k)
__device__ __forceinline__ void issue_t3b(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t sa = smem_u32(smem + kOffShi);
  const uint32_t slot = smem_u32(smem + ((c & 1) ? kOffSlot1 : kOffSlot0));
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ss(tbase + kColO, kmaj_desc(sa, kk), kmaj_desc(slot, kk), id, kk > 0 ? 1u : 0u);
}

// T4  S += Delta'_hi^T K + Delta'_lo^T K   (M=128 v, N=128 k, K=64 t; A from TMEM)
__device__ __forceinline__ void issue_t4(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id_upd = make_idesc(128, 128, 1, 0, 1);
  const uint32_t slot = smem_u32(smem + ((c & 1) ? kOffSlot1 : kOffSlot0));
  const uint32_t colx = (c & 1) ? kColX1 : kColX0;
#pragma unroll
  for (int part = 0; part < 2; ++part)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ts(tbase + kColS, tbase + colx + 32 + 32 * part + 8 * kk,
                   make_sdesc_sw128(slot + 8192 + kk * 2048, 16384, 1024), id_upd, 1u);
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_prefill_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base_shared;

  const int warp = warp_id();
  const int lane = lane_id();
  const int unit = blockIdx.x;
  const int order = unit / p.hv;
  const int h = unit - order * p.hv;
  const int seq = p.seq_order ? p.seq_order[order] : order;
  const int kh = h % p.hk;
  const int tok0 = p.cu_seqlens[seq];
  const int len = p.cu_seqlens[seq + 1] - tok0;
  const int nchunks = len > 0 ? (len + kC - 1) / kC : 0;
  ChunkParams* params = reinterpret_cast<ChunkParams*>(smem + kOffParams);
  float* scratch = reinterpret_cast<float*>(smem + kOffScratch);
  const size_t state_off = (static_cast<size_t>(seq) * p.hv + h) * kD * kD;

  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    uint64_t* all = reinterpret_cast<uint64_t*>(&bars);
    for (int i = 0; i < static_cast<int>(sizeof(Barriers) / 8); ++i) mbar_init(&all[i], 1);
    mbar_init(&drain_bar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.qk_read[i], 128);
      mbar_init(&bars.g_ready[i], 32);
      mbar_init(&bars.prep1[i], 64);
      mbar_init(&bars.wneg[i], 128);
      mbar_init(&bars.da_done[i], 128);
      mbar_init(&bars.s_ready[i], 128);
      mbar_init(&bars.p_ready[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&tmem_base_shared, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_shared;
  if (threadIdx.x == 0) GDN_TRACE(19, 0);

  if (nchunks == 0) {
    // empty sequence: final state = initial state
    if (warp < 4) {
      const int v = threadIdx.x;
      for (int kk = 0; kk < kD; kk += 4) {
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.state_in) val = *reinterpret_cast<const float4*>(p.state_in + state_off + v * kD + kk);
        *reinterpret_cast<float4*>(p.state_out + state_off + v * kD + kk) = val;
      }
    }
  } else if (warp < 4) {
    // =========================================================== state chain (lane = value row)
    const int v = threadIdx.x;
    const uint32_t lane_base = tmem_addr(tbase, warp * 32, 0);
    // --- initial state: hi/lo bf16 copies, TMEM S <- gamma_C(0) * S0
    bool ok = wait_c_warp(bars.g_ready, 0, p.status, kDevTimeoutPipe);
    if (ok) {
      const float gam = params[0].gamma_c;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[64];
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
          float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
          if (p.state_in) val = *reinterpret_cast<const float4*>(p.state_in + state_off + v * kD + half * 64 + j);
          sv[j] = __float_as_uint(val.x);
          sv[j + 1] = __float_as_uint(val.y);
          sv[j + 2] = __float_as_uint(val.z);
          sv[j + 3] = __float_as_uint(val.w);
        }
        store_state_half(smem, v, half, sv);
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
        tmem_st32(lane_base + kColS + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_st32(lane_base + kColS + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      }
      fence_async_smem();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.s_ready[0]);
    }
    for (int c = 0; ok && c < nchunks; ++c) {
      const ChunkParams& pc = params[c & 1];
      const uint32_t colx = (c & 1) ? kColX1 : kColX0;
      // --- (one thread) T3a: the state-dependent part of Delta, as soon as S(c) and W(c) exist
      if (v == 0 && wait_c(bars.s_ready, c, p.status, kDevTimeoutPipe) &&
          wait_c(bars.wneg, c, p.status, kDevTimeoutPipe)) {
        tc_fence_after();
        issue_t3a(tbase, smem, c);
        umma_commit(&bars.delta[c & 1]);
        GDN_TRACE(13, c);
      }
      // --- Delta pass: Delta^T (fp32) -> bf16 Delta, Delta' = e^{G_C - G} Delta as hi + lo
      if (!wait_c_warp(bars.delta, c, p.status, kDevTimeoutMma)) { ok = false; break; }
      tc_fence_after();
      if (v == 0) GDN_TRACE(0, c);
      {
        uint32_t d[64];
        tmem_ld64(lane_base + colx, d);
        uint32_t pk[32], hi[32], lo[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d0 = __uint_as_float(d[2 * j]);
          const float d1 = __uint_as_float(d[2 * j + 1]);
          pk[j] = pack_bf16x2(d0, d1);
          split_pack(d0 * pc.egr[2 * j], d1 * pc.egr[2 * j + 1], hi[j], lo[j]);
        }
        tmem_st32(lane_base + colx, pk);
        tmem_st32(lane_base + colx + 32, hi);
        tmem_st32(lane_base + colx + 64, lo);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(&bars.da_done[c & 1]);
      if (v == 0) GDN_TRACE(1, c);
      // --- (one thread) T4: the state update
      if (v == 0 && wait_c(bars.da_done, c, p.status, kDevTimeoutPipe)) {
        tc_fence_after();
        issue_t4(tbase, smem, c);
        umma_commit(&bars.snew[c & 1]);
        GDN_TRACE(14, c);
      }
      // --- state pass: S (fp32) -> hi/lo bf16 copies for the next chunk, pre-scale by its decay
      //     (the copies are overwritten in place: T3b, the other reader, must have completed)
      if (!wait_c_warp(bars.snew, c, p.status, kDevTimeoutMma)) { ok = false; break; }
      if (!wait_c_warp(bars.t3b, c, p.status, kDevTimeoutMma)) { ok = false; break; }
      tc_fence_after();
      if (v == 0) GDN_TRACE(2, c);
      const bool last = (c == nchunks - 1);
      float gam = 1.0f;
      if (!last) {
        if (!wait_c_warp(bars.g_ready, c + 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
        gam = params[(c + 1) & 1].gamma_c;
      }
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[64];
        tmem_ld64(lane_base + kColS + half * 64, sv);
        if (v == 0 && half == 0) GDN_TRACE(21, c);
        if (last) {
          float* dst = p.state_out + state_off + v * kD + half * 64;
#pragma unroll
          for (int j = 0; j < 64; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1]),
                                                              __uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3]));
        } else {
          store_state_half(smem, v, half, sv);
#pragma unroll
          for (int j = 0; j < 64; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
          tmem_st32(lane_base + kColS + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_st32(lane_base + kColS + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        }
      }
      if (!last) {
        fence_async_smem();
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars.s_ready[(c + 1) & 1]);
        if (v == 0) GDN_TRACE(3, c);
      }
    }
  } else if (warp < 8) {
    // =========================================================== operand warps
    const int r = threadIdx.x - 128;  // TMEM lane / row owned by this thread
    const uint32_t lane_base = tmem_addr(tbase, (warp & 3) * 32, 0);
    bool ok = true;
    for (int c = 0; ok && c < nchunks; ++c) {
      ChunkParams& pc = params[c & 1];
      // --- (1) decay prefix sums for chunk c (warp 4)
      if (warp == 4) {
        if (c >= 2 && !wait_c_warp(bars.da_done, c - 2, p.status, kDevTimeoutPipe)) { ok = false; break; }
        const int n_valid = min(kC, len - c * kC);
        const int t0 = 2 * lane, t1 = 2 * lane + 1;
        const size_t base = static_cast<size_t>(tok0 + c * kC);
        const float ga = t0 < n_valid ? p.g[(base + t0) * p.hv + h] : 0.0f;
        const float gb = t1 < n_valid ? p.g[(base + t1) * p.hv + h] : 0.0f;
        const float ba = t0 < n_valid ? p.beta[(base + t0) * p.hv + h] : 0.0f;
        const float bb = t1 < n_valid ? p.beta[(base + t1) * p.hv + h] : 0.0f;
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
        __syncwarp();
        mbar_arrive(&bars.g_ready[c & 1]);
        if (lane == 0) GDN_TRACE(18, c);
      }
      // --- (2a) QK / KK read-out: e^G-scaled Q (in place), L rows -> solve scratch; P row kept
      //          in registers until the P tile is free
      bool ready = wait_c_warp(bars.qk_done, c, p.status, kDevTimeoutMma);
      if (ready) ready = wait_c_warp(bars.g_ready, c, p.status, kDevTimeoutPipe);
      if (ready && c >= 1) ready = wait_c_warp(bars.w_done, c - 1, p.status, kDevTimeoutMma);  // T tiles free
      if (!ready) { ok = false; break; }
      tc_fence_after();
      uint32_t prow[32];
      if (r == 0) GDN_TRACE(4, c);
      {
        uint32_t row[64];
        tmem_ld64(lane_base + kColQK, row);
        if (r == 0) GDN_TRACE(22, c);
        if (r < 64) {
          const int t = r;
          const float gt = pc.g2[t];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int s0 = 2 * j, s1 = 2 * j + 1;
            const float p0 = s0 <= t ? __uint_as_float(row[s0]) * ex2_approx(gt - pc.g2[s0]) : 0.0f;
            const float p1 = s1 <= t ? __uint_as_float(row[s1]) * ex2_approx(gt - pc.g2[s1]) : 0.0f;
            prow[j] = pack_bf16x2(p0, p1);
          }
          // Q row t lives in rows 0..63 of the stacked slot, 2 boxes of 64 columns
          uint8_t* slot = smem + ((c & 1) ? kOffSlot1 : kOffSlot0);
          const float eg = pc.eg[t];
#pragma unroll
          for (int bx = 0; bx < 2; ++bx) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint4* ptr = reinterpret_cast<uint4*>(slot + bx * 16384 + t * 128 + ((j ^ (t & 7)) << 4));
              uint4 val = *ptr;
              uint32_t* w = reinterpret_cast<uint32_t*>(&val);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 b2 = *reinterpret_cast<__nv_bfloat162*>(&w[e]);
                const float2 f = __bfloat1622float2(b2);
                w[e] = pack_bf16x2(f.x * eg, f.y * eg);
              }
              *ptr = val;
            }
          }
        } else {
          const int t = r - 64;
          const float gt = pc.g2[t];
          const float bt = pc.beta[t];
#pragma unroll
          for (int s = 0; s < 64; ++s)
            scratch[s * 64 + t] = s < t ? bt * ex2_approx(gt - pc.g2[s]) * __uint_as_float(row[s]) : 0.0f;
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars.qk_read[c & 1]);
      if (r == 0) GDN_TRACE(5, c);
      // --- (3) W pass: W^T (lane = key row k) -> -W as [k][t], hi and lo bf16 tiles
      ready = wait_c_warp(bars.w_done, c, p.status, kDevTimeoutMma);
      if (ready && c >= 1) ready = wait_c_warp(bars.delta, c - 1, p.status, kDevTimeoutMma);  // W tiles free
      if (!ready) { ok = false; break; }
      tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t row[32];
        tmem_ld32(lane_base + kColW + 32 * half, row);
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          split_pack(-__uint_as_float(row[2 * j]), -__uint_as_float(row[2 * j + 1]), hi[j], lo[j]);
        store_half_row_sw128(smem + kOffWhi, r, half, hi);
        store_half_row_sw128(smem + kOffWlo, r, half, lo);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars.wneg[c & 1]);
      if (r == 0) GDN_TRACE(6, c);
      // --- (4) output pass of the previous chunk, then the P tile of this chunk (single buffer:
      //         the previous chunk's P V MMA has completed once its output is ready)
      if (c >= 1) {
        if (!wait_c_warp(bars.o_done, c - 1, p.status, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        output_pass(p, lane_base, tok0, len, c - 1, h, r);
        if (r == 0) GDN_TRACE(7, c - 1);
        tc_fence_before();
      }
      // --- (5) T3b: O^T = S_hi (e^G Q)^T once all 128 threads have read the O region out and
      //         the state copy of chunk c exists
      if (!named_sync_and(2, 128, true)) { ok = false; break; }
      if (r == 0 && wait_c(bars.s_ready, c, p.status, kDevTimeoutPipe)) {
        tc_fence_after();
        issue_t3b(tbase, smem, c);
        umma_commit(&bars.t3b[c & 1]);
        GDN_TRACE(15, c);
      }
      if (r < 64) store_row_sw128(smem + kOffP, r, prow);
      fence_async_smem();
      mbar_arrive(&bars.p_ready[c & 1]);
      if (r == 0) GDN_TRACE(8, c);
    }
    if (ok && wait_c_warp(bars.o_done, nchunks - 1, p.status, kDevTimeoutMma)) {
      tc_fence_after();
      output_pass(p, lane_base, tok0, len, nchunks - 1, h, r);
    }
  } else if (warp < 10) {
    // =========================================================== triangular solve
    // That = (I + L)^-1, one column per thread (warps 8, 9), by 16-row blocks: for block B the
    // thread starts from e_j, subtracts the contributions of the already-solved rows
    // (left-looking, sum_{s < 16B} L[r][s] x_s) and finishes the block by right-looking forward
    // substitution.  Only 16 accumulators are live; solved rows go to an fp32 column buffer in
    // shared memory (each thread reads back only its own column).  A warp skips the blocks above
    // its first column (x = 0 there).  Column j then becomes row j of the MN-major ([s][t]) tiles
    // T = That diag(beta) and T diag(e^G), each as hi + lo.
    const int tid = threadIdx.x - 256;
    const int j = tid;                 // column
    const int wfirst = tid & ~31;      // first column of this warp
    float* xbuf = reinterpret_cast<float*>(smem + kOffTGhi);  // That[r][j] at xbuf[r * 64 + j]
    bool ok = true;
    for (int c = 0; ok && c < nchunks; ++c) {
      const bool ready = wait_c(bars.qk_read, c, p.status, kDevTimeoutPipe);
      // the two warps leave together or not at all (they meet at named barriers below)
      if (!named_sync_and(1, 64, ready)) { ok = false; break; }
      if (tid == 0) GDN_TRACE(9, c);
      const ChunkParams& pc = params[c & 1];
#pragma unroll
      for (int B = 0; B < 4; ++B) {
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = (16 * B + i == j) ? 1.0f : 0.0f;
        if (16 * B + 15 >= wfirst) {  // warp-uniform
          // left-looking: rows of the previous blocks (x_s = 0 for s < j)
#pragma unroll 2
          for (int s0 = wfirst; s0 < 16 * B; ++s0) {
            const float xs = xbuf[s0 * 64 + j];
            const float4* lc = reinterpret_cast<const float4*>(scratch + s0 * 64 + 16 * B);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 l = lc[q];
              acc[4 * q + 0] = fmaf(-l.x, xs, acc[4 * q + 0]);
              acc[4 * q + 1] = fmaf(-l.y, xs, acc[4 * q + 1]);
              acc[4 * q + 2] = fmaf(-l.z, xs, acc[4 * q + 2]);
              acc[4 * q + 3] = fmaf(-l.w, xs, acc[4 * q + 3]);
            }
          }
          // right-looking inside the block (L[r][t] = 0 for r <= t)
#pragma unroll
          for (int tt = 0; tt < 15; ++tt) {
            const float xt = acc[tt];
            const float* lc = scratch + (16 * B + tt) * 64 + 16 * B;
#pragma unroll
            for (int i4 = (tt + 1) & ~3; i4 < 16; i4 += 4) {
              const float4 l = *reinterpret_cast<const float4*>(lc + i4);
              acc[i4 + 0] = fmaf(-l.x, xt, acc[i4 + 0]);
              acc[i4 + 1] = fmaf(-l.y, xt, acc[i4 + 1]);
              acc[i4 + 2] = fmaf(-l.z, xt, acc[i4 + 2]);
              acc[i4 + 3] = fmaf(-l.w, xt, acc[i4 + 3]);
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) xbuf[(16 * B + i) * 64 + j] = acc[i];
      }
      float x[64];
#pragma unroll
      for (int r = 0; r < 64; ++r) x[r] = xbuf[r * 64 + j];
      named_sync(1, 64);  // L and every column are in registers: the tiles may overwrite both
      const float w0 = pc.beta[j];
      const float w1 = w0 * pc.eg[j];
#pragma unroll
      for (int q = 0; q < 2; ++q) {  // q = 0: T, q = 1: T diag(e^G)
        const float w = q ? w1 : w0;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) split_pack(x[32 * hf + 2 * i] * w, x[32 * hf + 2 * i + 1] * w, hi[i], lo[i]);
          store_half_row_sw128(smem + (q ? kOffTGhi : kOffThi), j, hf, hi);
          store_half_row_sw128(smem + (q ? kOffTGlo : kOffTlo), j, hf, lo);
        }
      }
      fence_async_smem();
      if (tid == 0) GDN_TRACE(10, c);
      mbar_arrive(&bars.prep1[c & 1]);
    }
  } else if (warp == kWarpTma) {
    // =========================================================== TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int row = tok0 + c * kC;
        // the slot of chunk c-2 is free once its state pass ran: T1-T4 and T3b have completed
        if (c >= 2 && !wait_c(bars.s_ready, c - 1, p.status, kDevTimeoutPipe)) break;
        uint8_t* slot = smem + ((c & 1) ? kOffSlot1 : kOffSlot0);
        mbar_arrive_expect_tx(&bars.in_full[c & 1], kSlotBytes);
        GDN_TRACE(17, c);
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_3d(slot + bx * 16384, &map_q, &bars.in_full[c & 1], bx * 64, kh, row);
          tma_load_3d(slot + bx * 16384 + 8192, &map_k, &bars.in_full[c & 1], bx * 64, kh, row);
        }
        if (c >= 1 && !wait_c(bars.v_free, c - 1, p.status, kDevTimeoutPipe)) break;
        mbar_arrive_expect_tx(&bars.v_full[c & 1], 16384);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_3d(smem + kOffV + bx * 8192, &map_v, &bars.v_full[c & 1], bx * 64, h, row);
        issued = c + 1;
      }
      // before the CTA retires, let the last loads land (bounded; a no-op on the normal path)
      for (int c = max(0, issued - 2); c < issued; ++c) {
        mbar_drain(&bars.in_full[c & 1], (c >> 1) & 1);
        mbar_drain(&bars.v_full[c & 1], (c >> 1) & 1);
      }
    }
  } else {
    // =========================================================== MMA issuer (polling)
    // Groups per chunk c (the state-dependent groups T3a/T4 are issued by the state-chain warps,
    // T3b by the operand warps):
    //   T1  [Q;K] K^T                                                   -> QK region
    //   T2  W^T = K^T (TG_hi + TG_lo)^T ; Delta^T = V^T (T_hi + T_lo)^T  -> W region, X slot
    //   T5  O^T += Delta^T P^T
    // This thread polls the hand-off barriers (non-blocking) and issues whichever group is ready.
    if (lane == 0 && nchunks > 0) {
      const uint32_t id_qk = make_idesc(128, 64, 1, 0, 0);    // [Q;K] K^T
      const uint32_t id_mnmn = make_idesc(128, 64, 1, 1, 1);  // A MN-major (K^T, V^T), B MN-major (T tiles [s][t])
      const uint32_t id_dp = make_idesc(128, 64, 1, 0, 0);    // A TMEM, B K-major (P [t][s])
      const uint32_t a_thi = smem_u32(smem + kOffThi), a_tlo = smem_u32(smem + kOffTlo);
      const uint32_t a_tghi = smem_u32(smem + kOffTGhi), a_tglo = smem_u32(smem + kOffTGlo);
      const uint32_t a_v = smem_u32(smem + kOffV), a_p = smem_u32(smem + kOffP);
      int n1 = 0, n2 = 0, n5 = 0;
      const int N = nchunks;
      unsigned long long idle_since = 0;
      uint32_t idle_polls = 0;
      while (n5 < N) {
        bool issued = false;
        if (n5 < n2 && test_c(bars.t3b, n5) && test_c(bars.da_done, n5) && test_c(bars.p_ready, n5)) {
          // T5: O^T += Delta^T P^T
          const int c = n5;
          tc_fence_after();
          const uint32_t colx = (c & 1) ? kColX1 : kColX0;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ts(tbase + kColO, tbase + colx + 8 * kk, make_sdesc_sw128(a_p + kk * 32, 16, 1024), id_dp, 1u);
          umma_commit(&bars.o_done[c & 1]);
          GDN_TRACE(16, c);
          ++n5;
          issued = true;
        } else if (n2 < n1 && n2 < n5 + 2 && test_c(bars.prep1, n2) && test_c(bars.v_full, n2) &&
                   (n2 == 0 || test_c(bars.wneg, n2 - 1)) && (n2 < 2 || test_c(bars.snew, n2 - 2))) {
          // T2: W^T = K^T (TG_hi + TG_lo)^T ; Delta^T = V^T T_hi^T + V^T T_lo^T
          // (the X slot of chunk c was last read by T4(c-2) and T5(c-2))
          const int c = n2;
          tc_fence_after();
          const uint32_t slot = smem_u32(smem + ((c & 1) ? kOffSlot1 : kOffSlot0));
          const uint32_t colx = (c & 1) ? kColX1 : kColX0;
#pragma unroll
          for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ss(tbase + kColW, make_sdesc_sw128(slot + 8192 + kk * 2048, 16384, 1024),
                           make_sdesc_sw128((part ? a_tglo : a_tghi) + kk * 2048, 16384, 1024), id_mnmn,
                           (part > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ss(tbase + colx, make_sdesc_sw128(a_v + kk * 2048, 8192, 1024),
                           make_sdesc_sw128((part ? a_tlo : a_thi) + kk * 2048, 16384, 1024), id_mnmn,
                           (part > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&bars.w_done[c & 1]);
          umma_commit(&bars.v_free[c & 1]);
          GDN_TRACE(12, c);
          ++n2;
          issued = true;
        } else if (n1 < N && n1 <= n2 + 1 && test_c(bars.in_full, n1) && (n1 == 0 || test_c(bars.qk_read, n1 - 1))) {
          // T1: [Q;K] K^T
          const int c = n1;
          tc_fence_after();
          const uint32_t slot = smem_u32(smem + ((c & 1) ? kOffSlot1 : kOffSlot0));
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ss(tbase + kColQK, kmaj_desc(slot, kk), kmaj_desc(slot + 8192, kk), id_qk, kk > 0 ? 1u : 0u);
          umma_commit(&bars.qk_done[c & 1]);
          GDN_TRACE(11, c);
          ++n1;
          issued = true;
        }
        if (issued) {
          idle_polls = 0;
        } else if ((++idle_polls & 255u) != 0u) {
          __nanosleep(32);  // leave issue slots and shared-memory bandwidth to the other warps
        } else {
          // every 256 empty polls: give up after kWaitTimeoutNs without progress, or as soon as
          // another warp of the CTA has reported a timeout
          const unsigned long long now = global_timer_ns();
          if (idle_polls == 256u) idle_since = now;
          if (cta_abort_flag() != 0u) break;
          if (now - idle_since > kWaitTimeoutNs) {
            record_status(p.status, kDevTimeoutPipe);
            cta_abort_flag() = 1u;
            break;
          }
        }
      }
      // every MMA issued by this thread completes before TMEM is released (bounded)
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace gdn
}  // namespace tokmix

extern "C" int tokmix_gdn_prefill(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  const float* initial_state, void* out, float* final_state,
                                  const int32_t* cu_seqlens_dev, const int32_t* seq_order_dev, int num_seqs,
                                  int total_tokens, int heads_k, int heads_v, int head_dim_k, int head_dim_v,
                                  float scale, int io_dtype, uint32_t* status, void* stream) {
  using namespace tokmix;
  using namespace tokmix::gdn;
  if (!q || !k || !v || !g || !beta || !out || !final_state || !cu_seqlens_dev)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: null pointer argument");
  if (num_seqs < 0 || total_tokens < 0 || heads_k <= 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: negative or zero size");
  if (heads_v % heads_k != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: heads_v (%d) must be a multiple of heads_k (%d)",
                heads_v, heads_k);
  if (head_dim_k != kD || head_dim_v != kD)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill: head dims must be 128 (got %d, %d)", head_dim_k,
                head_dim_v);
  if (io_dtype != TOKMIX_DTYPE_BF16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill: only bf16 q/k/v/out are supported by the kernel");
  if (!std::isfinite(scale)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: scale must be finite");
  if (status == nullptr)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: a device status word is required");
  for (const void* ptr : {q, k, v, static_cast<const void*>(initial_state), static_cast<const void*>(final_state)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: tensors must be 16-byte aligned");
  if (num_seqs == 0) return TOKMIX_OK;
  if (const int rc = check_device()) return rc;
  const long long units = static_cast<long long>(num_seqs) * heads_v;
  if (units > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill: too many (sequence, head) units");

  // 3-D tensor maps over (dim, head, token); box = 64 columns x 1 head x 64 tokens.
  const uint64_t rows = static_cast<uint64_t>(total_tokens > 0 ? total_tokens : 1);
  CUtensorMap mq, mk, mv;
  {
    uint64_t dims_k[3] = {kD, static_cast<uint64_t>(heads_k), rows};
    uint64_t strides_k[2] = {kD * 2, static_cast<uint64_t>(heads_k) * kD * 2};
    uint64_t dims_v[3] = {kD, static_cast<uint64_t>(heads_v), rows};
    uint64_t strides_v[2] = {kD * 2, static_cast<uint64_t>(heads_v) * kD * 2};
    uint32_t box[3] = {64, 1, 64};
    if (!encode_tiled(&mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims_k, strides_k, box,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims_k, strides_k, box,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims_v, strides_v, box,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return TOKMIX_ERR_INVALID_ARGUMENT;
  }
  Params p{};
  p.g = g;
  p.beta = beta;
  p.state_in = initial_state;
  p.state_out = final_state;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.cu_seqlens = cu_seqlens_dev;
  p.seq_order = seq_order_dev;
  p.hk = heads_k;
  p.hv = heads_v;
  p.scale = scale;
  p.status = status;
  const int smem_bytes = kSmemBytes + 1024;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(&gdn_prefill_kernel), smem_bytes))
    return check_launch("tokmix_gdn_prefill: cudaFuncSetAttribute");
  gdn_prefill_kernel<<<static_cast<unsigned>(units), kThreads, smem_bytes, static_cast<cudaStream_t>(stream)>>>(
      mq, mk, mv, p);
  return check_launch("tokmix_gdn_prefill");
}

#ifdef TOKMIX_GDN_TRACE
extern "C" int tokmix_gdn_trace_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn;
  const int count = n < kTraceEvents * kTraceChunks ? n : kTraceEvents * kTraceChunks;
  return cudaMemcpyFromSymbol(host, g_trace, sizeof(unsigned long long) * count) == cudaSuccess ? count : -1;
}
#endif

// ---------------------------------------------------------------------------------------------
// Allocation-free entry point for equal-length batches.
//
// Some callers cannot allocate device memory when they run an op: a graph executor that plans
// every buffer ahead of time (the llama.cpp-style backends the reference's fp32 GDN interface is
// written for), or C / FFI callers without a device allocator.  They can hand us their inputs
// and outputs, but not the small scratch the kernel needs (the per-sequence token offsets and
// the device status word).  This entry point keeps that scratch in a file-scope device array.
namespace tokmix {
namespace gdn {
namespace noalloc {

constexpr int kMaxSeqs = 4095;  // largest batch this entry point accepts
// [0, 64): status word (word 0) + padding; [64, 64 + kMaxSeqs + 1): token offsets of the batch
static __device__ __align__(256) int32_t g_scratch[64 + kMaxSeqs + 1];

__global__ void fill_offsets(int32_t* offsets, int batch, int seqlen, uint32_t* status_to_clear) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i <= batch) offsets[i] = i * seqlen;
  if (i == 0 && status_to_clear != nullptr) *status_to_clear = 0u;
}

std::mutex g_mu;
int32_t* g_base[64] = {};  // device address of g_scratch, per device (set up once)

}  // namespace noalloc
}  // namespace gdn
}  // namespace tokmix

extern "C" int tokmix_gdn_prefill_noalloc(const void* q, const void* k, const void* v, const float* g,
                                          const float* beta, const float* initial_state, void* out,
                                          float* final_state, int batch, int seqlen, int heads_k, int heads_v,
                                          int head_dim_k, int head_dim_v, float scale, int io_dtype,
                                          uint32_t* status, void* stream) {
  using namespace tokmix;
  namespace na = tokmix::gdn::noalloc;
  if (batch < 0 || seqlen < 0) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_noalloc: negative size");
  if (batch > na::kMaxSeqs)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_noalloc: batch %d exceeds the maximum of %d",
                batch, na::kMaxSeqs);
  if (static_cast<long long>(batch) * seqlen > 0x7FFFFFFFll)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_noalloc: batch * seqlen exceeds 2^31 - 1");
  if (batch == 0) return TOKMIX_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(TOKMIX_ERR_DEVICE, "tokmix_gdn_prefill_noalloc: no usable current device");
  int32_t* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(na::g_mu);
    if (na::g_base[dev] == nullptr) {
      // set-up, once per device, with that device current: the host-side symbol is only a
      // stand-in, the kernels need the device address of this device's copy of the array
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, na::g_scratch);
      if (e != cudaSuccess)
        return fail(TOKMIX_ERR_DEVICE, "tokmix_gdn_prefill_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
      na::g_base[dev] = static_cast<int32_t*>(ptr);
    }
    base = na::g_base[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* st = status != nullptr ? status : reinterpret_cast<uint32_t*>(base);
  int32_t* offsets = base + 64;
  na::fill_offsets<<<(batch + 1 + 255) / 256, 256, 0, s>>>(offsets, batch, seqlen, status != nullptr ? nullptr : st);
  if (const int rc = check_launch("tokmix_gdn_prefill_noalloc")) return rc;
  return tokmix_gdn_prefill(q, k, v, g, beta, initial_state, out, final_state, offsets, nullptr, batch, batch * seqlen,
                            heads_k, heads_v, head_dim_k, head_dim_v, scale, io_dtype, st, stream);
}
