// gdn_prefill.cu -- chunked gated-delta-rule prefill for sm_100a (B200).
//
// Reference path replaced: kernels_optimized/qwen35moe_gdn_prefill.cu:683-1161 (precompute +
// chunk-scan kernels) behind qwen35moe_gdn_prefill_bf16tc (:1203-1264).  Maths: the fp32
// recurrence kernels/qwen35moe_gdn_prefill.cu:55-99 (value head h reads key head h % Hk,
// state layout [v][k], output computed with the updated state).
//
// Chunked form used here (C = 64 tokens, in-chunk cumulative log decay G_t, incoming state S0):
//   L_ts  = beta_t exp(G_t - G_s) (k_t . k_s)          s < t
//   T     = (I + L)^-1 diag(beta)                      (unit-lower inverse in fp32, 16x16 blocks)
//   W     = T diag(e^G) K                              (tensor core; T diag(e^G) as bf16 hi + lo)
//   Delta = T V - W S0^T                               (tensor core; T as hi + lo; W S0^T as the
//                                                       3-term product W_hi S_hi + W_lo S_hi + W_hi S_lo)
//   O     = scale (diag(e^G) Q S0^T + P Delta),  P_ts = exp(G_t - G_s)(q_t . k_s), s <= t
//   S     = e^{G_C} S0 + (diag(e^{G_C - G}) Delta)^T K (tensor core; Delta' split hi + lo)
// Every contraction is an M=128 tcgen05 MMA because the CTA keeps the VALUE dimension on the
// 128 TMEM lanes ("transposed" products: Delta^T, O^T, S with lane = value row; W^T with
// lane = key row).  The fp32 state and its hi + lo bf16 copies (the A operand of the next
// chunk's products) never leave TMEM between chunks.  The hi/lo splits keep every product that
// feeds the state at ~16 significant bits, so the fp32 final state stays within 1e-3 relative of
// the fp32 recurrence even when the decay is weak.
//
// One CTA processes one (sequence, value head) unit, all its chunks in order.  Only the state
// chain is sequential: Delta(c) -> S(c+1) -> Delta(c+1).  Everything that does not depend on the
// state (decay sums, Q K^T / K K^T, the triangular solve, W) is prepared for chunk c+1 while the
// chain works on chunk c.  Warp roles (384 threads):
//   warps 0-3   state chain, thread = value row: issues the state-dependent MMAs, Delta pass
//               (Delta -> bf16 operands in TMEM), state pass (S -> hi/lo copies, decay for the
//               next chunk), initial / final state; thread 0 also issues every TMA load
//   warps 4-7   operands, each warp polling on its own: decay prefix sums (warp 4), Q K^T / K K^T
//               read-out (P tile, e^G-scaled Q in place, rows of L), output pass (O^T -> global)
//   warps 8-11  triangular solve (16x16 blocks), T / T diag(e^G) tiles, W pass (W^T -> -W
//               tiles); thread 0 issues the preparation MMAs (Q K^T, W)
// Hand-off barriers are two-slot arrays indexed by chunk parity (the Q/K ring has three).  Every
// producer of chunk c+2's event causally follows every waiter of chunk c's event, so no waiter
// can fall two phases behind (argued next to each barrier below).  All waits are bounded.
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
constexpr int kSlots = 3;  // Q/K chunk tiles in flight

// TMEM columns (512 allocated)
constexpr uint32_t kColS = 0;      // state S[v][k] fp32, 128 cols
constexpr uint32_t kColShi = 128;  // state hi copy, bf16 pairs along k, 64 cols
constexpr uint32_t kColSlo = 192;  // state lo copy
constexpr uint32_t kColX = 256;    // Delta^T fp32 (64 cols), then Delta'hi | Delta'lo | Delta bf16 (32 each)
constexpr uint32_t kColO = 352;    // O^T fp32, 64 cols
constexpr uint32_t kColQW = 416;   // Q K^T (lanes 0-63) / K K^T (lanes 64-127), later W^T (lane = key row)

// shared memory layout (bytes; every MMA tile starts on a 1024-byte boundary)
constexpr int kSlotBytes = 32768;                  // stacked [Q;K] chunk tile: 2 boxes of 128 rows x 128 B
constexpr int kOffSlots = 0;                       //   rows 0-63 of a box: Q (scaled in place to scale e^G Q)
                                                   //   rows 64-127: K
constexpr int kOffV = kSlots * kSlotBytes;         // V chunk tile: 2 boxes of 64 rows x 128 B
constexpr int kOffP = kOffV + 16384;               // P [t][s] bf16, 2 x 8 KB (chunk parity)
constexpr int kOffT = kOffP + 16384;               // T hi [s][t] (8 KB), T lo (8 KB)
constexpr int kLds = 68;                           // fp32 row stride of the solve matrices
constexpr int kOffL = kOffT + 16384;               // L fp32 [t][s] (row stride kLds); after the
                                                   //   solve: T diag(e^G) hi [s][t], lo (8 KB each)
constexpr int kOffX = kOffL + 64 * kLds * 4;       // (I + L)^-1 fp32 [t][s] (row stride kLds)
constexpr int kOffW = kOffX + 64 * kLds * 4;       // -W hi as [k][t] (16 KB), -W lo (16 KB)
constexpr int kOffStage = kOffW + 32768;           // output staging, 4 warps x 32 tokens x 64 B
constexpr int kOffParams = kOffStage + 8192;
constexpr int kParamsBytes = 1280;
constexpr int kSmemBytes = kOffParams + 2 * kParamsBytes;
static_assert(kOffL % 1024 == 0 && kOffX % 1024 == 0 && kOffW % 1024 == 0, "tile alignment");
static_assert(kSmemBytes + 1024 + 512 <= 227 * 1024, "shared memory budget");

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

// Hand-off barriers.  Event of chunk c lives in slot c & 1 (in_full: c % 3) and completes the
// slot's (c >> 1)-th (c / 3-th) phase.
struct Barriers {
  uint64_t in_full[kSlots];  // TMA Q/K(c) landed.   waiter: solve t0 (T1).  next phase needs T4(c)
  uint64_t v_full[2];        // TMA V(c) landed.     waiter: chain t0 (T3).  V(c+2) issued after T3(c+1)
  uint64_t qk_done[2];       // T1(c) complete.      waiters: operand warps; T1(c+2) follows readout(c+1)
  uint64_t qk_read[2];       // read-out(c) done (128). waiters: solve; readout(c+2) follows T1(c+2) <- solve(c+1)
  uint64_t g_ready[2];       // decay sums(c) (32).  waiters: operand warps, chain; scan(c+2) follows output(c)
  uint64_t w_done[2];        // T2(c) complete.      waiters: solve; T2(c+2) follows their W pass(c+1)
  uint64_t w_ready[2];       // W/T tiles(c) (128).  waiter: chain t0; W pass(c+2) follows T3(c+1)
  uint64_t x_ready[2];       // T3(c) complete.      waiters: chain, solve; T3(c+2) follows both
  uint64_t s_new[2];         // T3b(c), T4(c) complete. waiters: chain
  uint64_t o_done[2];        // T5(c) complete.      waiters: operand warps, chain t0
  uint64_t o_read[2];        // O(c) read out (128). waiter: chain t0 (T3b(c+1))
  uint64_t drain[2];         // retirement of the two MMA-issuing threads
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

// K-major tile of 2 boxes (16 KB apart): descriptor of the 16-element k step kk
__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}

__device__ __forceinline__ uint32_t slot_addr(const uint8_t* smem, int c) {
  return smem_u32(smem + kOffSlots + (c % kSlots) * kSlotBytes);
}

// T1  [Q;K] K^T   (M=128 rows of the stacked tile, N=64 keys s, K=128)
__device__ __forceinline__ void issue_t1(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t slot = slot_addr(smem, c);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ss(tbase + kColQW, kmaj_desc(slot, kk), kmaj_desc(slot + 8192, kk), id, kk > 0 ? 1u : 0u);
}

// T2  W^T = K^T (TG_hi + TG_lo)^T   (M=128 k, N=64 t, K=64 s; both operands MN-major)
__device__ __forceinline__ void issue_t2(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 1, 1);
  const uint32_t kt = slot_addr(smem, c) + 8192;
  const uint32_t tg = smem_u32(smem + kOffL);
#pragma unroll
  for (int part = 0; part < 2; ++part)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ss(tbase + kColQW, make_sdesc_sw128(kt + kk * 2048, 16384, 1024),
                   make_sdesc_sw128(tg + part * 8192 + kk * 2048, 16384, 1024), id, (part > 0 || kk > 0) ? 1u : 0u);
}

// T3  Delta^T = V^T (T_hi + T_lo)^T + S_hi (-W_hi)^T + S_lo (-W_hi)^T + S_hi (-W_lo)^T
//     (M=128 v, N=64 t; the state terms take S from TMEM)
__device__ __forceinline__ void issue_t3(uint32_t tbase, const uint8_t* smem) {
  const uint32_t id_v = make_idesc(128, 64, 1, 1, 1);  // A = V^T MN-major, B = T [s][t] MN-major
  const uint32_t id_s = make_idesc(128, 64, 1, 0, 1);  // A = S (TMEM), B = -W [k][t] MN-major
  const uint32_t a_v = smem_u32(smem + kOffV), a_t = smem_u32(smem + kOffT), a_w = smem_u32(smem + kOffW);
#pragma unroll
  for (int part = 0; part < 2; ++part)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ss(tbase + kColX, make_sdesc_sw128(a_v + kk * 2048, 8192, 1024),
                   make_sdesc_sw128(a_t + part * 8192 + kk * 2048, 16384, 1024), id_v, (part > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
  for (int term = 0; term < 3; ++term) {
    const uint32_t sa = tbase + (term == 1 ? kColSlo : kColShi);
    const uint32_t wb = a_w + (term == 2 ? 16384 : 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16_ts(tbase + kColX, sa + 8 * kk, make_sdesc_sw128(wb + kk * 2048, 16384, 1024), id_s, 1u);
  }
}

// T3b  O^T = S_hi (scale e^G Q)^T   (M=128 v, N=64 t, K=128 k; A from TMEM)
__device__ __forceinline__ void issue_t3b(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t slot = slot_addr(smem, c);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ts(tbase + kColO, tbase + kColShi + 8 * kk, kmaj_desc(slot, kk), id, kk > 0 ? 1u : 0u);
}

// T4  S += Delta'_hi^T K + Delta'_lo^T K   (M=128 v, N=128 k, K=64 t; A from TMEM)
__device__ __forceinline__ void issue_t4(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 128, 1, 0, 1);
  const uint32_t kt = slot_addr(smem, c) + 8192;
#pragma unroll
  for (int part = 0; part < 2; ++part)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ts(tbase + kColS, tbase + kColX + 32 * part + 8 * kk, make_sdesc_sw128(kt + kk * 2048, 16384, 1024),
                   id, 1u);
}

// T5  O^T += Delta^T (scale P)^T   (M=128 v, N=64 t, K=64 s; A from TMEM, B = P [t][s] K-major)
__device__ __forceinline__ void issue_t5(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t a_p = smem_u32(smem + kOffP + (c & 1) * 8192);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    umma_bf16_ts(tbase + kColO, tbase + kColX + 64 + 8 * kk, make_sdesc_sw128(a_p + kk * 32, 16, 1024), id, 1u);
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_prefill_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
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
  const int N = len > 0 ? (len + kC - 1) / kC : 0;
  ChunkParams* params = reinterpret_cast<ChunkParams*>(smem + kOffParams);
  const size_t state_off = (static_cast<size_t>(seq) * p.hv + h) * kD * kD;

  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    uint64_t* all = reinterpret_cast<uint64_t*>(&bars);
    for (int i = 0; i < static_cast<int>(sizeof(Barriers) / 8); ++i) mbar_init(&all[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.qk_read[i], 128);
      mbar_init(&bars.g_ready[i], 32);
      mbar_init(&bars.w_ready[i], 128);
      mbar_init(&bars.o_read[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_shared, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_shared;
  if (threadIdx.x == 0) GDN_TRACE(19, 0);

  if (N == 0) {
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
    const uint32_t lb = tmem_addr(tbase, warp * 32, 0);
    int qk_issued = 0, v_issued = 0;
    auto load_qk = [&](int c) {  // thread 0 only
      const int s = c % kSlots;
      uint8_t* slot = smem + kOffSlots + s * kSlotBytes;
      mbar_arrive_expect_tx(&bars.in_full[s], kSlotBytes);
      for (int bx = 0; bx < 2; ++bx) {
        tma_load_3d(slot + bx * 16384, &map_q, &bars.in_full[s], bx * 64, kh, tok0 + c * kC);
        tma_load_3d(slot + bx * 16384 + 8192, &map_k, &bars.in_full[s], bx * 64, kh, tok0 + c * kC);
      }
      qk_issued = c + 1;
    };
    auto load_v = [&](int c) {  // thread 0 only
      mbar_arrive_expect_tx(&bars.v_full[c & 1], 16384);
      for (int bx = 0; bx < 2; ++bx)
        tma_load_3d(smem + kOffV + bx * 8192, &map_v, &bars.v_full[c & 1], bx * 64, h, tok0 + c * kC);
      v_issued = c + 1;
    };
    if (v == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      for (int c = 0; c < kSlots && c < N; ++c) load_qk(c);
      load_v(0);
    }
    // --- initial state: hi/lo copies and S <- gamma(0) S0
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
        store_split32<0>(lb + kColShi + 32 * half, lb + kColSlo + 32 * half, sv);
        store_split32<32>(lb + kColShi + 32 * half + 16, lb + kColSlo + 32 * half + 16, sv);
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
        tmem_st32(lb + kColS + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_st32(lb + kColS + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      }
      tmem_wait_st();
    }
    tc_fence_before();
    ok = named_sync_and(1, 128, ok);
    for (int c = 0; ok && c < N; ++c) {
      // --- (thread 0) T3 as soon as the W/T tiles and V of chunk c exist and T5(c-1) has read
      //     the X region; then T3b once the output pass has read O(c-1)
      if (v == 0) {
        bool r = wait_c(bars.w_ready, c, p.status, kDevTimeoutPipe) &&
                 wait_c(bars.v_full, c, p.status, kDevTimeoutTma) &&
                 (c == 0 || wait_c(bars.o_done, c - 1, p.status, kDevTimeoutMma));
        if (r) {
          tc_fence_after();
          issue_t3(tbase, smem);
          umma_commit(&bars.x_ready[c & 1]);
          GDN_TRACE(0, c);
        }
        if (r && c >= 1) r = wait_c(bars.o_read, c - 1, p.status, kDevTimeoutPipe);
        if (r) {
          tc_fence_after();
          issue_t3b(tbase, smem, c);
        }
      }
      // --- Delta pass: Delta^T (fp32) -> Delta'hi | Delta'lo | Delta bf16
      // (every exit from this loop goes through a named_sync_and, so the four warps leave together)
      const bool xr = wait_c_warp(bars.x_ready, c, p.status, kDevTimeoutMma);
      tc_fence_after();
      if (xr && v == 0) {
        GDN_TRACE(1, c);
        if (c + 1 < N) load_v(c + 1);  // V(c) has been read by T3(c)
      }
      if (xr) {
        const ChunkParams& pc = params[c & 1];
        uint32_t d[64];
        tmem_ld64(lb + kColX, d);
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          split_pack(__uint_as_float(d[2 * j]) * pc.egr[2 * j], __uint_as_float(d[2 * j + 1]) * pc.egr[2 * j + 1],
                     hi[j], lo[j]);
        tmem_st32(lb + kColX, hi);
        tmem_st32(lb + kColX + 32, lo);
#pragma unroll
        for (int j = 0; j < 32; ++j) hi[j] = pack_bf16x2(__uint_as_float(d[2 * j]), __uint_as_float(d[2 * j + 1]));
        tmem_st32(lb + kColX + 64, hi);
        tmem_wait_st();
      }
      tc_fence_before();
      if (!named_sync_and(1, 128, xr)) { ok = false; break; }
      if (v == 0) {
        GDN_TRACE(2, c);
        tc_fence_after();
        issue_t4(tbase, smem, c);
        umma_commit(&bars.s_new[c & 1]);
        issue_t5(tbase, smem, c);
        umma_commit(&bars.o_done[c & 1]);
      }
      // --- state pass: S(c+1) -> hi/lo copies, pre-scaled fp32 state for the next update
      const bool last = (c == N - 1);
      bool sr = wait_c_warp(bars.s_new, c, p.status, kDevTimeoutMma);
      tc_fence_after();
      if (sr && v == 0) {
        GDN_TRACE(3, c);
        if (c + kSlots < N) load_qk(c + kSlots);  // every reader of Q/K(c) has completed
      }
      float gam = 1.0f;
      if (sr && !last) {
        sr = wait_c_warp(bars.g_ready, c + 1, p.status, kDevTimeoutPipe);
        gam = params[(c + 1) & 1].gamma_c;
      }
#pragma unroll 1
      for (int half = 0; sr && half < 2; ++half) {
        uint32_t sv[64];
        tmem_ld64(lb + kColS + half * 64, sv);
        if (last) {
          float* dst = p.state_out + state_off + v * kD + half * 64;
#pragma unroll
          for (int j = 0; j < 64; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1]),
                                                              __uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3]));
        } else {
          store_split32<0>(lb + kColShi + 32 * half, lb + kColSlo + 32 * half, sv);
          store_split32<32>(lb + kColShi + 32 * half + 16, lb + kColSlo + 32 * half + 16, sv);
#pragma unroll
          for (int j = 0; j < 64; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
          tmem_st32(lb + kColS + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_st32(lb + kColS + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        }
      }
      if (!last) {
        tmem_wait_st();
        tc_fence_before();
        if (!named_sync_and(1, 128, sr)) { ok = false; break; }
        if (v == 0) GDN_TRACE(4, c);
      }
    }
    if (v == 0) {
      // before the CTA retires: this thread's MMAs and TMA loads have landed (bounded; no-ops on
      // the normal path)
      umma_commit(&bars.drain[0]);
      mbar_drain(&bars.drain[0], 0);
      for (int c = max(0, qk_issued - kSlots); c < qk_issued; ++c)
        mbar_drain(&bars.in_full[c % kSlots], (c / kSlots) & 1);
      if (v_issued > 0) mbar_drain(&bars.v_full[(v_issued - 1) & 1], ((v_issued - 1) >> 1) & 1);
    }
  } else if (warp < 8) {
    // =========================================================== operand warps
    // Each warp polls on its own (lane 0 tests, the warp follows): output pass of chunk co once
    // T5(co) is done, decay sums of chunk cg (warp 4), read-out of chunk cr once T1(cr) is done.
    const int r = threadIdx.x - 128;  // TMEM lane / row owned by this thread
    const int wq = warp & 3;
    const uint32_t lb = tmem_addr(tbase, wq * 32, 0);
    float* Ls = reinterpret_cast<float*>(smem + kOffL);
    uint8_t* stage = smem + kOffStage + wq * 2048;
    int cr = 0, co = 0, cg = (warp == 4) ? 0 : N;
    // decay inputs of chunk cg, two tokens per lane, loaded one chunk ahead (warp 4)
    float ga = 0.f, gb = 0.f, ba = 0.f, bb = 0.f;
    auto load_g = [&](int c) {
      const int n_valid = min(kC, len - c * kC);
      const int t0 = 2 * lane, t1 = 2 * lane + 1;
      const size_t base = static_cast<size_t>(tok0 + c * kC);
      ga = t0 < n_valid ? p.g[(base + t0) * p.hv + h] : 0.0f;
      gb = t1 < n_valid ? p.g[(base + t1) * p.hv + h] : 0.0f;
      ba = t0 < n_valid ? p.beta[(base + t0) * p.hv + h] : 0.0f;
      bb = t1 < n_valid ? p.beta[(base + t1) * p.hv + h] : 0.0f;
    };
    if (warp == 4) load_g(0);
    unsigned long long idle_since = 0;
    uint32_t idle_polls = 0;
    while (co < N) {
      bool did = false;
      // (1) output pass of chunk co
      if (co < cr && __shfl_sync(0xffffffffu, lane == 0 ? test_c(bars.o_done, co) : false, 0)) {
        tc_fence_after();
        if (r == 0) GDN_TRACE(7, co);
        uint32_t o[64];
        tmem_ld64(lb + kColO, o);
        tc_fence_before();
        mbar_arrive(&bars.o_read[co & 1]);
        const int nv = min(kC, len - co * kC);
        __nv_bfloat16* dst = p.out + (static_cast<size_t>(tok0 + co * kC) * p.hv + h) * kD + wq * 32;
        const size_t tstride = static_cast<size_t>(p.hv) * kD;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          // stage[i][v] for 32 tokens i, 16-byte chunks XOR-swizzled by (i >> 1) & 3
#pragma unroll
          for (int i = 0; i < 32; ++i)
            *reinterpret_cast<__nv_bfloat16*>(stage + i * 64 + ((((lane >> 3) ^ (i >> 1)) & 3) << 4) +
                                              ((lane & 7) << 1)) = __float2bfloat16_rn(__uint_as_float(o[32 * hf + i]));
          __syncwarp();
          const int t = 32 * hf + lane;
          if (t < nv) {
            const uint8_t* src = stage + lane * 64;
            uint4* g = reinterpret_cast<uint4*>(dst + t * tstride);
#pragma unroll
            for (int j = 0; j < 4; ++j) g[j] = *reinterpret_cast<const uint4*>(src + (((j ^ (lane >> 1)) & 3) << 4));
          }
          __syncwarp();
        }
        if (r == 0) GDN_TRACE(8, co);
        ++co;
        did = true;
      } else if (cg < N && cg <= co + 1) {
        // (2) decay prefix sums of chunk cg (warp 4).  Its params slot held chunk cg-2, whose
        //     last readers (Delta pass, state pass) finished before T5(cg-2) and so before the
        //     output pass of cg-2 that this warp has done.
        ChunkParams& pc = params[cg & 1];
        const int n_valid = min(kC, len - cg * kC);
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
        __syncwarp();
        mbar_arrive(&bars.g_ready[cg & 1]);
        if (lane == 0) GDN_TRACE(15, cg);
        ++cg;
        if (cg < N) load_g(cg);
        did = true;
      } else if (cr < N && cr <= co + 1 &&
                 __shfl_sync(0xffffffffu, lane == 0 ? (test_c(bars.qk_done, cr) && test_c(bars.g_ready, cr)) : false,
                             0)) {
        // (3) read-out of chunk cr: P row (scale folded in), scale e^G Q in place, L row.  The P
        //     slot was last read by T5(cr-2) (output pass cr-2 done); the L region by T2(cr-1),
        //     which completed before T1(cr) was issued.
        tc_fence_after();
        if (r == 0) GDN_TRACE(5, cr);
        const ChunkParams& pc = params[cr & 1];
        uint32_t row[64];
        tmem_ld64(lb + kColQW, row);
        if (r < 64) {
          const int t = r;
          const float gt = pc.g2[t];
          uint32_t prow[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int s0 = 2 * j, s1 = 2 * j + 1;
            const float p0 = s0 <= t ? __uint_as_float(row[s0]) * ex2_approx(gt - pc.g2[s0]) * p.scale : 0.0f;
            const float p1 = s1 <= t ? __uint_as_float(row[s1]) * ex2_approx(gt - pc.g2[s1]) * p.scale : 0.0f;
            prow[j] = pack_bf16x2(p0, p1);
          }
          store_row_sw128(smem + kOffP + (cr & 1) * 8192, t, prow);
          // Q row t lives in rows 0..63 of the stacked slot, 2 boxes of 64 columns
          uint8_t* slot = smem + kOffSlots + (cr % kSlots) * kSlotBytes;
          const float f = pc.eg[t] * p.scale;
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
                const float2 fl = __bfloat1622float2(b2);
                w[e] = pack_bf16x2(fl.x * f, fl.y * f);
              }
              *ptr = val;
            }
          }
        } else {
          const int t = r - 64;
          const float gt = pc.g2[t];
          const float bt = pc.beta[t];
          float* lrow = Ls + t * kLds;
#pragma unroll
          for (int s4 = 0; s4 < 64; s4 += 4) {
            float4 val;
            val.x = s4 + 0 < t ? bt * ex2_approx(gt - pc.g2[s4 + 0]) * __uint_as_float(row[s4 + 0]) : 0.0f;
            val.y = s4 + 1 < t ? bt * ex2_approx(gt - pc.g2[s4 + 1]) * __uint_as_float(row[s4 + 1]) : 0.0f;
            val.z = s4 + 2 < t ? bt * ex2_approx(gt - pc.g2[s4 + 2]) * __uint_as_float(row[s4 + 2]) : 0.0f;
            val.w = s4 + 3 < t ? bt * ex2_approx(gt - pc.g2[s4 + 3]) * __uint_as_float(row[s4 + 3]) : 0.0f;
            *reinterpret_cast<float4*>(lrow + s4) = val;
          }
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars.qk_read[cr & 1]);
        if (r == 0) GDN_TRACE(6, cr);
        ++cr;
        did = true;
      }
      if (did) {
        idle_polls = 0;
      } else if ((++idle_polls & 255u) != 0u) {
        __nanosleep(64);
      } else {
        // every 256 empty polls: give up after kWaitTimeoutNs without progress, or as soon as
        // another warp of the CTA has reported a timeout
        const unsigned long long now = global_timer_ns();
        if (idle_polls == 256u) idle_since = now;
        const bool stop = cta_abort_flag() != 0u || now - idle_since > kWaitTimeoutNs;
        if (__shfl_sync(0xffffffffu, stop, 0)) {
          if (cta_abort_flag() == 0u && lane == 0) {
            record_status(p.status, kDevTimeoutPipe);
            cta_abort_flag() = 1u;
          }
          break;
        }
      }
    }
  } else {
    // =========================================================== triangular solve and W
    // X = (I + L)^-1 by 16x16 blocks: the four diagonal blocks by forward substitution (one
    // column per thread), then block rows i = 1..3 as X[i, <i] = -D_i (L[i, <i] X[<i, <i]).
    // X's diagonal blocks hold explicit zeros above the diagonal; the blocks above the block
    // diagonal are never read.
    const int tid = threadIdx.x - 256;
    const uint32_t lb = tmem_addr(tbase, (warp & 3) * 32, 0);
    float* Ls = reinterpret_cast<float*>(smem + kOffL);
    float* Xs = reinterpret_cast<float*>(smem + kOffX);
    bool ok = true;
    if (tid == 0) {
      ok = mbar_wait(&bars.in_full[0], 0, p.status, kDevTimeoutTma);
      if (ok) {
        tc_fence_after();
        issue_t1(tbase, smem, 0);
        umma_commit(&bars.qk_done[0]);
        GDN_TRACE(14, 0);
      }
    }
    for (int c = 0; c < N; ++c) {
      const bool ready = wait_c(bars.qk_read, c, p.status, kDevTimeoutPipe);
      if (!named_sync_and(3, 128, ready && ok)) { ok = false; break; }
      if (tid == 0) GDN_TRACE(9, c);
      // --- diagonal blocks D_b = (I + L_bb)^-1, column j per thread
      if (tid < 64) {
        const int b = tid >> 4, j = tid & 15;
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
        for (int i = 0; i < 16; ++i) Xs[(16 * b + i) * kLds + 16 * b + j] = acc[i];
      }
      named_sync(3, 128);
      // --- block rows 1..3; thread = (row rr of the block row, column pair cg of each block)
      {
        const int rr = tid >> 3, cg = tid & 7;
#pragma unroll
        for (int i = 1; i < 4; ++i) {
          float2 y[3];
          const float* lrow = Ls + (16 * i + rr) * kLds;
#pragma unroll
          for (int cb = 0; cb < i; ++cb) {
            const int c0 = 16 * cb + 2 * cg;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int k4 = 16 * cb; k4 < 16 * i; k4 += 4) {
              const float4 l = *reinterpret_cast<const float4*>(lrow + k4);
              const float2 x0 = *reinterpret_cast<const float2*>(Xs + (k4 + 0) * kLds + c0);
              const float2 x1 = *reinterpret_cast<const float2*>(Xs + (k4 + 1) * kLds + c0);
              const float2 x2 = *reinterpret_cast<const float2*>(Xs + (k4 + 2) * kLds + c0);
              const float2 x3 = *reinterpret_cast<const float2*>(Xs + (k4 + 3) * kLds + c0);
              a0 = fmaf(l.x, x0.x, a0);
              a1 = fmaf(l.x, x0.y, a1);
              a0 = fmaf(l.y, x1.x, a0);
              a1 = fmaf(l.y, x1.y, a1);
              a0 = fmaf(l.z, x2.x, a0);
              a1 = fmaf(l.z, x2.y, a1);
              a0 = fmaf(l.w, x3.x, a0);
              a1 = fmaf(l.w, x3.y, a1);
            }
            y[cb] = make_float2(a0, a1);
          }
          // Y = L[i, <i] X[<i, <i] goes to X's block row i (not read by this step)
#pragma unroll
          for (int cb = 0; cb < i; ++cb) *reinterpret_cast<float2*>(Xs + (16 * i + rr) * kLds + 16 * cb + 2 * cg) = y[cb];
          named_sync(3, 128);
          float dr[16];
#pragma unroll
          for (int m4 = 0; m4 < 16; m4 += 4) {
            const float4 d4 = *reinterpret_cast<const float4*>(Xs + (16 * i + rr) * kLds + 16 * i + m4);
            dr[m4] = d4.x;
            dr[m4 + 1] = d4.y;
            dr[m4 + 2] = d4.z;
            dr[m4 + 3] = d4.w;
          }
          float2 z[3];
#pragma unroll
          for (int cb = 0; cb < i; ++cb) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              const float2 ym = *reinterpret_cast<const float2*>(Xs + (16 * i + m) * kLds + 16 * cb + 2 * cg);
              a0 = fmaf(dr[m], ym.x, a0);
              a1 = fmaf(dr[m], ym.y, a1);
            }
            z[cb] = make_float2(-a0, -a1);
          }
          named_sync(3, 128);
#pragma unroll
          for (int cb = 0; cb < i; ++cb) *reinterpret_cast<float2*>(Xs + (16 * i + rr) * kLds + 16 * cb + 2 * cg) = z[cb];
          named_sync(3, 128);
        }
      }
      if (tid == 0) GDN_TRACE(10, c);
      // --- T = X diag(beta) and T diag(e^G) as MN-major hi/lo tiles (row s, tokens t of one
      //     half).  The T tiles and the W tiles were last read by T3(c-1).
      const bool free_tiles = (c == 0) || wait_c(bars.x_ready, c - 1, p.status, kDevTimeoutMma);
      if (!named_sync_and(3, 128, free_tiles)) { ok = false; break; }
      {
        const ChunkParams& pc = params[c & 1];
        const int s = tid & 63, half = tid >> 6;
        float xv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int t = 32 * half + i;
          xv[i] = t >= s ? Xs[t * kLds + s] : 0.0f;
        }
        const float w0 = pc.beta[s];
        const float w1 = w0 * pc.eg[s];
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // q = 0: T, q = 1: T diag(e^G) (over the dead L)
          const float w = q ? w1 : w0;
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) split_pack(xv[2 * i] * w, xv[2 * i + 1] * w, hi[i], lo[i]);
          uint8_t* tile = smem + (q ? kOffL : kOffT);
          store_half_row_sw128(tile, s, half, hi);
          store_half_row_sw128(tile + 8192, s, half, lo);
        }
      }
      fence_async_smem();
      named_sync(3, 128);
      if (tid == 0) {
        tc_fence_after();
        issue_t2(tbase, smem, c);
        umma_commit(&bars.w_done[c & 1]);
        GDN_TRACE(12, c);
      }
      // --- W pass: W^T (lane = key row k) -> -W as [k][t], hi and lo tiles
      const bool wready = wait_c_warp(bars.w_done, c, p.status, kDevTimeoutMma);
      if (wready) {
        tc_fence_after();
        uint32_t row[64];
        tmem_ld64(lb + kColQW, row);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            split_pack(-__uint_as_float(row[32 * half + 2 * j]), -__uint_as_float(row[32 * half + 2 * j + 1]), hi[j],
                       lo[j]);
          store_half_row_sw128(smem + kOffW, tid, half, hi);
          store_half_row_sw128(smem + kOffW + 16384, tid, half, lo);
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars.w_ready[c & 1]);
      }
      // every thread has read W^T out of the QW region: T1(c+1) may overwrite it
      if (!named_sync_and(3, 128, wready)) { ok = false; break; }
      if (tid == 0) {
        GDN_TRACE(13, c);
        const int n = c + 1;
        if (n < N) {
          ok = mbar_wait(&bars.in_full[n % kSlots], (n / kSlots) & 1, p.status, kDevTimeoutTma);
          if (ok) {
            tc_fence_after();
            issue_t1(tbase, smem, n);
            umma_commit(&bars.qk_done[n & 1]);
            GDN_TRACE(14, n);
          }
        }
      }
    }
    if (tid == 0) {
      umma_commit(&bars.drain[1]);
      mbar_drain(&bars.drain[1], 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
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
