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
//   warps 0-3   state chain, thread = value row: Delta pass (Delta -> bf16 operands in TMEM),
//               state pass (S -> hi/lo copies, decay for the next chunk), initial / final
//               state; thread 0 issues the state-dependent MMAs and every TMA load
//   warps 4-7   operands, each warp polling on its own: K K^T / Q K^T read-out (warps 4-5: rows
//               of L; warps 6-7: P tile and e^G-scaled Q in place), output pass (O^T ->
//               global), decay prefix sums (warp 7)
//   warps 8-11  triangular solve, T / T diag(e^G) tiles, W pass (W^T -> -W tiles); thread 0
//               issues the preparation MMAs (Q K^T, W, T V)
// Hand-off barriers are two-slot arrays indexed by chunk parity (the Q/K ring has three).  Every
// producer of chunk c+2's event causally follows every waiter of chunk c's event, so no waiter
// can fall two phases behind (argued next to each barrier below).  All waits are bounded.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "gdn_common.cuh"
#include "host_common.h"

namespace tokmix {
namespace gdn {

constexpr int kThreads = 384;
constexpr int kSlots = 3;  // Q/K chunk tiles in flight

// TMEM columns (512 allocated)
constexpr uint32_t kColS = 0;      // state S[v][k] fp32, 128 cols
constexpr uint32_t kColShi = 128;  // state hi copy, bf16 pairs along k, 64 cols
constexpr uint32_t kColSlo = 192;  // state lo copy
constexpr uint32_t kColX = 256;    // Delta^T as two fp32 halves (64 + 64 cols, summed by the Delta pass),
                                   // then Delta'hi | Delta'lo | Delta bf16 (32 cols each)
constexpr uint32_t kColO = 384;    // O^T fp32, 64 cols
constexpr uint32_t kColQW = 448;   // K K^T (lanes 0-63) / Q K^T (lanes 64-127), later W^T (lane = key row)

// shared memory layout (bytes; every MMA tile starts on a 1024-byte boundary)
constexpr int kSlotBytes = 32768;                  // stacked [K;Q] chunk tile: 2 boxes of 128 rows x 128 B
constexpr int kOffSlots = 0;
constexpr int kKRows = 0;                          //   rows 0-63 of a box: K
constexpr int kQRows = 8192;                       //   rows 64-127: Q (scaled in place to scale e^G Q)
constexpr int kOffV = kSlots * kSlotBytes;         // V chunk tile: 2 boxes of 64 rows x 128 B
constexpr int kOffP = kOffV + 16384;               // P [t][s] bf16, 2 x 8 KB (chunk parity)
constexpr int kOffT = kOffP + 16384;               // T hi [s][t] (8 KB), T lo (8 KB)
constexpr int kOffL = kOffT + 16384;               // L fp32 [t][s] (row stride kLds); after the
                                                   //   solve: T diag(e^G) hi [s][t], lo (8 KB each)
constexpr int kOffX = kOffL + 64 * kLds * 4;       // (I + L)^-1 fp32 [t][s] (row stride kLds)
constexpr int kOffW = kOffX + 64 * kLds * 4;       // -W hi as [k][t] (16 KB), -W lo (16 KB)
constexpr int kOffParams = kOffW + 32768;
constexpr int kSmemBytes = kOffParams + 2 * kParamsBytes;
static_assert(kOffL % 1024 == 0 && kOffX % 1024 == 0 && kOffW % 1024 == 0, "tile alignment");
static_assert(kSmemBytes + 1024 + 512 <= 227 * 1024, "shared memory budget");

struct Params {
  const float* g;
  const float* beta;
  const float* state_in;
  float* state_out;
  __nv_bfloat16* out;
  const int32_t* cu_seqlens;
  const int32_t* seq_order;
  int hk, hv;
  int num_seqs, total_tokens;
  float scale;
  uint32_t* status;
  GateSource gates;  // a == null: g and beta as given
  int l2norm;        // normalise the q and k rows as they are staged (before T1)
  float l2norm_eps;
};

// Hand-off barriers.  Event of chunk c lives in slot c & 1 (in_full: c % 3) and completes the
// slot's (c >> 1)-th (c / 3-th) phase.  For each: who waits, and why the event of chunk c+2
// cannot complete before every waiter has seen chunk c's.
struct Barriers {
  uint64_t in_full[kSlots];  // TMA Q/K(c).          solve t0 (T1).          Q/K(c+3) is loaded after T4(c)
  uint64_t v_full[2];        // TMA V(c).            solve t0 (TV).          V(c+2) is loaded after TV(c+1)
  uint64_t qk_done[2];       // T1(c).               operand warps.          T1(c+2) follows their read-out(c+1)
  uint64_t qk_ld[2];         // QK(c) loaded (128).  solve t0 (T2).          read-out(c+2) follows T2(c+1)
  uint64_t l_ready[2];       // L(c) rows (64).      solve.                  read-out(c+2) follows T1(c+2) <- solve(c+1)
  uint64_t pq_ready[2];      // P(c), e^G Q (64).    chain t0 (T3b, T5).     read-out(c+2) follows output pass(c) <- T5(c)
  uint64_t g_ready[2];       // decay sums(c) (32).  operand warps, chain.   scan(c+2) follows output pass(c)
  uint64_t w_done[2];        // T2(c).               solve.                  T2(c+2) follows their W pass(c+1)
  uint64_t w_ready[2];       // W/T tiles(c) (128).  chain t0 (state terms). W pass(c+2) follows x_ready(c+1)
  uint64_t tv_done[2];       // TV(c).               chain t0.               TV(c+2) follows o_done(c+1)
  uint64_t x_ready[2];       // state terms(c).      chain, solve.           state terms(c+2) follow both
  uint64_t s_new[2];         // T4(c).               chain.
  uint64_t o_done[2];        // T3b(c), T5(c).       operand warps, chain, solve t0.  T5(c+2) follows all
  uint64_t o_read[2];        // O(c) read (128).     chain t0 (T3b(c+1)).    output pass(c+2) follows T5(c+2)
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
// The whole warp arrives once (lane 0, count 32) after its lanes' prior writes are ordered by
// __syncwarp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31u) == 0u) mbar_arrive_count(bar, 32);
}

// Optional phase trace (build with -DTOKMIX_GDN_TRACE): SM clock stamps of CTA 0, indexed
// by event and chunk, read back with tokmix_gdn_trace_read().  Compiled out otherwise.
#ifdef TOKMIX_GDN_TRACE
constexpr int kTraceChunks = 64;
constexpr int kTraceEvents = 48;
__device__ unsigned long long g_trace[kTraceEvents * kTraceChunks];
#define GDN_TRACE(ev, c)                                                                          \
  do {                                                                                            \
    if (blockIdx.x == 0 && (c) < kTraceChunks) g_trace[(ev) * kTraceChunks + (c)] = clock64();   \
  } while (0)
#else
#define GDN_TRACE(ev, c) \
  do {                   \
  } while (0)
#endif

__device__ __forceinline__ uint32_t slot_addr(const uint8_t* smem, int c) {
  return smem_u32(smem + kOffSlots + (c % kSlots) * kSlotBytes);
}

// T1  [K;Q] K^T   (M=128 rows of the stacked tile, N=64 keys s, K=128)
__device__ __forceinline__ void issue_t1(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t slot = slot_addr(smem, c);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ss(tbase + kColQW, kmaj_desc(slot, kk, 16384), kmaj_desc(slot + kKRows, kk, 16384), id, kk > 0 ? 1u : 0u);
}

// T2  W^T = K^T (TG_hi + TG_lo)^T   (M=128 k, N=64 t, K=64 s; both operands MN-major)
__device__ __forceinline__ void issue_t2(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 1, 1);
  const uint32_t kt = slot_addr(smem, c) + kKRows;
  const uint32_t tg = smem_u32(smem + kOffL);
#pragma unroll
  for (int part = 0; part < 2; ++part)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ss(tbase + kColQW, make_sdesc_sw128(kt + kk * 2048, 16384, 1024),
                   make_sdesc_sw128(tg + part * 8192 + kk * 2048, 16384, 1024), id, (part > 0 || kk > 0) ? 1u : 0u);
}

// TV  [U_hi^T | U_lo^T] = V^T [T_hi | T_lo]^T   (M=128 v, N=128 (two 64-token halves), K=64 s)
__device__ __forceinline__ void issue_tv(uint32_t tbase, const uint8_t* smem) {
  const uint32_t id = make_idesc(128, 128, 1, 1, 1);  // A = V^T MN-major, B = T [s][t] MN-major, 2 chunks
  const uint32_t a_v = smem_u32(smem + kOffV), a_t = smem_u32(smem + kOffT);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    umma_bf16_ss(tbase + kColX, make_sdesc_sw128(a_v + kk * 2048, 8192, 1024),
                 make_sdesc_sw128(a_t + kk * 2048, 8192, 1024), id, kk > 0 ? 1u : 0u);
}

// state terms  X += S_hi [-W_hi | -W_lo]^T  (N=128) ;  X[:, 0:64] += S_lo (-W_hi)^T  (N=64)
//   (M=128 v, K=128 k; A = S from TMEM, B = -W [k][t] MN-major, hi and lo tiles 16 KB apart)
__device__ __forceinline__ void issue_state_terms(uint32_t tbase, const uint8_t* smem) {
  const uint32_t id128 = make_idesc(128, 128, 1, 0, 1);
  const uint32_t id64 = make_idesc(128, 64, 1, 0, 1);
  const uint32_t a_w = smem_u32(smem + kOffW);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ts(tbase + kColX, tbase + kColShi + 8 * kk, make_sdesc_sw128(a_w + kk * 2048, 16384, 1024), id128, 1u);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ts(tbase + kColX, tbase + kColSlo + 8 * kk, make_sdesc_sw128(a_w + kk * 2048, 16384, 1024), id64, 1u);
}

// T3b  O^T = S_hi (scale e^G Q)^T   (M=128 v, N=64 t, K=128 k; A from TMEM)
__device__ __forceinline__ void issue_t3b(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 64, 1, 0, 0);
  const uint32_t slot = slot_addr(smem, c);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ts(tbase + kColO, tbase + kColShi + 8 * kk, kmaj_desc(slot + kQRows, kk, 16384), id, kk > 0 ? 1u : 0u);
}

// T4  S += Delta'_hi^T K + Delta'_lo^T K   (M=128 v, N=128 k, K=64 t; A from TMEM)
__device__ __forceinline__ void issue_t4(uint32_t tbase, const uint8_t* smem, int c) {
  const uint32_t id = make_idesc(128, 128, 1, 0, 1);
  const uint32_t kt = slot_addr(smem, c) + kKRows;
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
  // The scheduling order and the token offsets are device data the host does not read: a unit
  // whose entries are out of range sets TOKMIX_DEV_BAD_ARGS and touches no memory.
  const int seq_raw = p.seq_order ? p.seq_order[order] : order;
  const bool seq_ok = seq_raw >= 0 && seq_raw < p.num_seqs;
  const int seq = seq_ok ? seq_raw : 0;
  const int kh = h % p.hk;
  const long long t_begin = p.cu_seqlens[seq], t_end = p.cu_seqlens[seq + 1];
  const bool bad = !seq_ok || t_begin < 0 || t_end < t_begin || t_end > p.total_tokens;
  const int tok0 = bad ? 0 : static_cast<int>(t_begin);
  const int len = bad ? 0 : static_cast<int>(t_end - t_begin);
  const int N = len > 0 ? (len + kC - 1) / kC : 0;
  ChunkParams* params = reinterpret_cast<ChunkParams*>(smem + kOffParams);
  const size_t state_off = (static_cast<size_t>(seq) * p.hv + h) * kD * kD;

  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    uint64_t* all = reinterpret_cast<uint64_t*>(&bars);
    for (int i = 0; i < static_cast<int>(sizeof(Barriers) / 8); ++i) mbar_init(&all[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.qk_ld[i], 128);
      mbar_init(&bars.l_ready[i], 64);
      mbar_init(&bars.pq_ready[i], 64);
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

  if (bad && threadIdx.x == 0) record_status(p.status, kDevBadArgs);
  if (N == 0) {
    // empty sequence: final state = initial state
    if (warp < 4 && !bad) {
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
        tma_load_3d(slot + bx * 16384 + kQRows, &map_q, &bars.in_full[s], bx * 64, kh, tok0 + c * kC);
        tma_load_3d(slot + bx * 16384 + kKRows, &map_k, &bars.in_full[s], bx * 64, kh, tok0 + c * kC);
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
      // --- (thread 0) state terms once W(c) exists and T V(c) is in the X region
      //     (every exit from this loop goes through a named_sync_and, so the four warps leave together)
      if (v == 0) {
        const bool r = wait_c(bars.w_ready, c, p.status, kDevTimeoutPipe) &&
                       wait_c(bars.tv_done, c, p.status, kDevTimeoutMma);
        if (r) {
          if (c + 1 < N) load_v(c + 1);  // V(c) has been read by TV(c)
          tc_fence_after();
          GDN_TRACE(28, c);
          issue_state_terms(tbase, smem);
          umma_commit(&bars.x_ready[c & 1]);
          GDN_TRACE(0, c);
        }
      }
      // --- Delta pass: X halves (fp32) -> Delta'hi | Delta'lo | Delta bf16
      if (v == 64) GDN_TRACE(40, c);
      const bool xr = wait_c_warp(bars.x_ready, c, p.status, kDevTimeoutMma);
      if (v == 64) GDN_TRACE(41, c);
      tc_fence_after();
      if (xr) {
        if (v == 0) GDN_TRACE(1, c);
        const ChunkParams& pc = params[c & 1];
        uint32_t d[64];
        tmem_ld64(lb + kColX, d);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t e[32];
          tmem_ld32(lb + kColX + 64 + 32 * hf, e);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            d[32 * hf + j] = __float_as_uint(__uint_as_float(d[32 * hf + j]) + __uint_as_float(e[j]));
        }
        if (v == 0) GDN_TRACE(18, c);
        // (every fp32 column is in registers, so the bf16 operands may overwrite the X region)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const int t = 32 * hf + 2 * j;
            const float4 e4 = *reinterpret_cast<const float4*>(&pc.egr[t]);
            split_pack(__uint_as_float(d[t]) * e4.x, __uint_as_float(d[t + 1]) * e4.y, hi[j], lo[j]);
            split_pack(__uint_as_float(d[t + 2]) * e4.z, __uint_as_float(d[t + 3]) * e4.w, hi[j + 1], lo[j + 1]);
          }
          tmem_st16(lb + kColX + 16 * hf, hi);
          tmem_st16(lb + kColX + 32 + 16 * hf, lo);
        }
        {
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pk[j] = pack_bf16x2(__uint_as_float(d[2 * j]), __uint_as_float(d[2 * j + 1]));
          tmem_st32(lb + kColX + 64, pk);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      if (!named_sync_and(1, 128, xr)) { ok = false; break; }
      if (v == 0) {
        GDN_TRACE(2, c);
        tc_fence_after();
        issue_t4(tbase, smem, c);
        umma_commit(&bars.s_new[c & 1]);
        // T3b and T5 (output of chunk c) once P(c) and e^G Q(c) exist and O(c-1) has been read
        if (wait_c(bars.pq_ready, c, p.status, kDevTimeoutPipe) &&
            (c == 0 || wait_c(bars.o_read, c - 1, p.status, kDevTimeoutPipe))) {
          tc_fence_after();
          issue_t3b(tbase, smem, c);
          GDN_TRACE(31, c);
          issue_t5(tbase, smem, c);
          umma_commit(&bars.o_done[c & 1]);
        }
      }
      // --- state pass: S(c+1) -> hi/lo copies, pre-scaled fp32 state for the next update.  The
      //     copies are overwritten only after T3b(c), their last reader, has completed (o_done).
      const bool last = (c == N - 1);
      if (v == 64) GDN_TRACE(42, c);
      bool sr = wait_c_warp(bars.s_new, c, p.status, kDevTimeoutMma);
      if (v == 64) GDN_TRACE(43, c);
      tc_fence_after();
      if (sr && v == 0) {
        GDN_TRACE(3, c);
        if (c + kSlots < N) load_qk(c + kSlots);  // every reader of Q/K(c) has completed (T3b(c) too)
      }
      float gam = 1.0f;
      if (sr && !last) {
        sr = wait_c_warp(bars.g_ready, c + 1, p.status, kDevTimeoutPipe) &&
             wait_c_warp(bars.o_done, c, p.status, kDevTimeoutMma);
        gam = params[(c + 1) & 1].gamma_c;
      }
#pragma unroll 1
      for (int qt = 0; sr && qt < 4; ++qt) {  // 32 state columns at a time
        uint32_t sv[32];
        tmem_ld32(lb + kColS + qt * 32, sv);
        if (v == 0 && qt == 0) GDN_TRACE(16, c);
        if (last) {
          float* dst = p.state_out + state_off + v * kD + qt * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1]),
                                                              __uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3]));
        } else {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            split_pack(__uint_as_float(sv[2 * j]), __uint_as_float(sv[2 * j + 1]), hi[j], lo[j]);
          tmem_st16(lb + kColShi + 16 * qt, hi);
          tmem_st16(lb + kColSlo + 16 * qt, lo);
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
          tmem_st32(lb + kColS + qt * 32, sv);
          if (v == 0 && qt == 1) GDN_TRACE(17, c);
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
    // Each warp polls on its own (lane 0 tests, the warp follows).  In order of priority: (warp
    // 7) decay sums of chunk cg; the read-out of chunk cr once T1(cr) is done (it gates the next
    // chunk's preparation); the output pass of chunk co once T5(co) is done.
    const int r = threadIdx.x - 128;  // TMEM lane / row owned by this thread
    const int wq = warp & 3;
    const uint32_t lb = tmem_addr(tbase, wq * 32, 0);
    float* Ls = reinterpret_cast<float*>(smem + kOffL);
    int cr = 0, co = 0;
    int cg = (warp == 7) ? 0 : N;
    // decay inputs of chunk cg, two tokens per lane, loaded one chunk ahead (warp 7)
    float ga = 0.f, gb = 0.f, ba = 0.f, bb = 0.f;
    auto load_g = [&](int c) {
      const int n_valid = min(kC, len - c * kC);
      const int t0 = 2 * lane, t1 = 2 * lane + 1;
      const size_t base = static_cast<size_t>(tok0 + c * kC);
      ga = gb = ba = bb = 0.0f;
      if (t0 < n_valid) load_gates(p.g, p.beta, p.gates, (base + t0) * p.hv + h, h, ga, ba);
      if (t1 < n_valid) load_gates(p.g, p.beta, p.gates, (base + t1) * p.hv + h, h, gb, bb);
    };
    if (warp == 7) load_g(0);
    unsigned long long idle_since = 0;
    uint32_t idle_polls = 0;
    while (co < N) {
      bool did = false;
      if (cg < N && cg <= co + 1) {
        // (1) decay prefix sums of chunk cg (warp 7).  Its params slot held chunk cg-2, whose
        //     last readers (Delta pass, state pass) finished before T5(cg-2) and so before the
        //     output pass of cg-2 that this warp has done.
        chunk_decay_params(params[cg & 1], ga, gb, ba, bb, min(kC, len - cg * kC), lane);
        __syncwarp();
        warp_arrive(&bars.g_ready[cg & 1]);
        if (lane == 0) GDN_TRACE(15, cg);
        ++cg;
        if (cg < N) load_g(cg);
        did = true;
      } else if (cr < N && cr <= co + 1 &&
                 __shfl_sync(0xffffffffu, lane == 0 ? (test_c(bars.qk_done, cr) && test_c(bars.g_ready, cr)) : false,
                             0)) {
        // (2) read-out of chunk cr.  The P slot was last read by T5(cr-2) (output pass cr-2 done);
        //     the L region by T2(cr-1), which completed before T1(cr) was issued.
        tc_fence_after();
        if (r == 0) GDN_TRACE(5, cr);
        if (r == 64) GDN_TRACE(36, cr);
        const ChunkParams& pc = params[cr & 1];
        uint32_t row[64];
        tmem_ld64(lb + kColQW, row);
        if (r == 96) GDN_TRACE(37, cr);
        if (r == 64) GDN_TRACE(39, cr);
        if (r == 32) GDN_TRACE(38, cr);
        tc_fence_before();
        if (r == 64) GDN_TRACE(44, cr);
        warp_arrive(&bars.qk_ld[cr & 1]);
        if (r == 64) GDN_TRACE(45, cr);
        if (r == 0) GDN_TRACE(24, cr);
        if (r == 64) GDN_TRACE(32, cr);
        if (r < 64) {
          l_row(row, pc, r, Ls);  // row r of L
          warp_arrive(&bars.l_ready[cr & 1]);
          if (r == 0) GDN_TRACE(33, cr);
        } else {
          // P row t (scale folded in), then scale e^G q_t in place
          const int t = r - 64;
          p_row(row, pc, t, p.scale, smem + kOffP + (cr & 1) * 8192);
          if (r == 64) GDN_TRACE(25, cr);
          scale_row_inplace(smem + kOffSlots + (cr % kSlots) * kSlotBytes + kQRows + t * 128, 16384, pc.eg[t] * p.scale);
          fence_async_smem();
          warp_arrive(&bars.pq_ready[cr & 1]);
        }
        if (r == 0) GDN_TRACE(6, cr);
        ++cr;
        did = true;
      } else if (co < cr && __shfl_sync(0xffffffffu, lane == 0 ? test_c(bars.o_done, co) : false, 0)) {
        // (3) output pass of chunk co (scale already folded into P and e^G Q)
        tc_fence_after();
        if (r == 0) GDN_TRACE(7, co);
        uint32_t o[64];
        tmem_ld64(lb + kColO, o);
        if (r == 0) GDN_TRACE(26, co);
        tc_fence_before();
        warp_arrive(&bars.o_read[co & 1]);
        // token pair (2i, 2i+1): the even lane of a lane pair stores (O[2i][v], O[2i][v+1]), the
        // odd lane (O[2i+1][v-1], O[2i+1][v]), one 4-byte store each
        const int nv = min(kC, len - co * kC);
        const bool odd = (lane & 1) != 0;
        const size_t tstride = static_cast<size_t>(p.hv) * kD;
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.out + (static_cast<size_t>(tok0 + co * kC) * p.hv + h) * kD +
                                                    (r & ~1)) + (odd ? tstride / 2 : 0);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = __uint_as_float(o[2 * i]), b = __uint_as_float(o[2 * i + 1]);
          const float other = __shfl_xor_sync(0xffffffffu, odd ? a : b, 1);
          const uint32_t packed = odd ? pack_bf16x2(other, b) : pack_bf16x2(a, other);
          if (2 * i + (odd ? 1 : 0) < nv) dst[i * tstride] = packed;
        }
        if (r == 0) GDN_TRACE(8, co);
        ++co;
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
    // X = (I + L)^-1 by recursive doubling over 16x16 blocks: the four diagonal blocks D_b by
    // forward substitution (one column per thread); the two 32x32 diagonal blocks E_0, E_1 from
    // X[2p+1, 2p] = -D_{2p+1} L[2p+1, 2p] D_{2p}; the lower 32x32 block as -E_1 L[1, 0] E_0.
    // Products are staged in X's strictly upper blocks, which nothing else reads; the diagonal
    // blocks hold explicit zeros above their diagonal.
    const int tid = threadIdx.x - 256;
    const uint32_t lb = tmem_addr(tbase, (warp & 3) * 32, 0);
    float* Ls = reinterpret_cast<float*>(smem + kOffL);
    float* Xs = reinterpret_cast<float*>(smem + kOffX);
    // qk_l2norm: the four warps normalise the 128 rows of chunk n's staged [K; Q] tile (thread =
    // row) once it has landed, before T1(n) -- its first reader
    auto normalize_slot = [&](int n) -> bool {
      bool landed = __all_sync(0xffffffffu, mbar_wait(&bars.in_full[n % kSlots], (n / kSlots) & 1, p.status,
                                                      kDevTimeoutTma));
      if (landed) {
        uint8_t* slot = smem + kOffSlots + (n % kSlots) * kSlotBytes;
        l2norm_row_sw128(slot + tid * 128, slot + 16384 + tid * 128, tid & 7, p.l2norm_eps);
        fence_async_smem();
      }
      return named_sync_and(3, 128, landed);
    };
    bool ok = true;
    if (p.l2norm) ok = normalize_slot(0);
    if (tid == 0 && ok) {
      ok = mbar_wait(&bars.in_full[0], 0, p.status, kDevTimeoutTma);
      if (ok) {
        tc_fence_after();
        issue_t1(tbase, smem, 0);
        umma_commit(&bars.qk_done[0]);
        GDN_TRACE(14, 0);
      }
    }
    // TV(c): V^T T^T into the X region once it is free (T4(c-1), T5(c-1) complete) and V(c) landed
    auto issue_tv_c = [&](int c) {  // thread 0 only
      tc_fence_after();
      issue_tv(tbase, smem);
      umma_commit(&bars.tv_done[c & 1]);
      GDN_TRACE(29, c);
    };
    for (int c = 0; c < N; ++c) {
      const bool ready = wait_c_warp(bars.l_ready, c, p.status, kDevTimeoutPipe);
      if (tid == 0) GDN_TRACE(34, c);
      if (tid == 64) GDN_TRACE(35, c);
      if (!named_sync_and(3, 128, ready && ok)) { ok = false; break; }
      if (tid == 0) GDN_TRACE(9, c);
      solve_inverse(Ls, PaddedRows{Xs}, tid, 3);
      if (tid == 0) GDN_TRACE(10, c);
      // --- T = X diag(beta) and T diag(e^G) as MN-major hi/lo tiles (row s, tokens t of one
      //     half).  The T tiles were last read by TV(c-1), the W tiles by the state terms(c-1).
      const bool free_tiles = (c == 0) || wait_c_warp(bars.x_ready, c - 1, p.status, kDevTimeoutMma);
      if (!named_sync_and(3, 128, free_tiles)) { ok = false; break; }
      if (tid == 0) GDN_TRACE(22, c);
      write_t_tiles(PaddedRows{Xs}, params[c & 1], tid, smem + kOffT, smem + kOffL);  // T diag(e^G) over the dead L
      if (tid == 0) GDN_TRACE(27, c);
      fence_async_smem();
      named_sync(3, 128);
      bool tv_issued = false;
      if (tid == 0) {
        // T2 once every operand warp has read Q K^T(c) out of the QW region
        if (wait_c(bars.qk_ld, c, p.status, kDevTimeoutPipe)) {
          tc_fence_after();
          GDN_TRACE(30, c);
          issue_t2(tbase, smem, c);
          umma_commit(&bars.w_done[c & 1]);
          GDN_TRACE(12, c);
        }
        if (test_c(bars.v_full, c) && (c == 0 || test_c(bars.o_done, c - 1))) {
          issue_tv_c(c);
          tv_issued = true;
        }
      }
      // --- W pass: W^T (lane = key row k) -> -W as [k][t], hi and lo tiles
      const bool wready = wait_c_warp(bars.w_done, c, p.status, kDevTimeoutMma);
      if (wready) {
        tc_fence_after();
        if (tid == 0) GDN_TRACE(23, c);
        uint32_t row[64];
        tmem_ld64(lb + kColQW, row);
        w_row(row, tid, smem + kOffW);
        fence_async_smem();
        tc_fence_before();
        warp_arrive(&bars.w_ready[c & 1]);
      }
      // every thread has read W^T out of the QW region: T1(c+1) may overwrite it
      if (!named_sync_and(3, 128, wready)) { ok = false; break; }
      if (p.l2norm && c + 1 < N && !normalize_slot(c + 1)) { ok = false; break; }
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
        if (ok && !tv_issued) {
          ok = wait_c(bars.v_full, c, p.status, kDevTimeoutTma) &&
               (c == 0 || wait_c(bars.o_done, c - 1, p.status, kDevTimeoutMma));
          if (ok) issue_tv_c(c);
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

namespace tokmix {
namespace gdn {

// Host-side argument checks of tokmix_gdn_prefill that do not depend on the token offsets (shared
// with the allocation-free entry point, which must reject a call before it touches its array).
static int validate_prefill_args(const char* who, const void* q, const void* k, const void* v, const float* g,
                                 const float* beta, const float* initial_state, const void* out,
                                 const float* final_state, int num_seqs, int total_tokens, int heads_k, int heads_v,
                                 int head_dim_k, int head_dim_v, float scale, int io_dtype,
                                 const tokmix_gdn_stage1* gates = nullptr) {
  if (!q || !k || !v || !out || !final_state || (!stage1_gates(gates) && (!g || !beta)))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: null pointer argument", who);
  if (const int rc = check_stage1(who, gates, false)) return rc;
  if (num_seqs < 0 || total_tokens < 0 || heads_k <= 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: negative or zero size", who);
  if (heads_v % heads_k != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: heads_v (%d) must be a multiple of heads_k (%d)", who, heads_v,
                heads_k);
  if (head_dim_k != kD || head_dim_v != kD)
    return fail(TOKMIX_ERR_UNSUPPORTED, "%s: head dims must be 128 (got %d, %d)", who, head_dim_k, head_dim_v);
  if (io_dtype != TOKMIX_DTYPE_BF16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "%s: only bf16 q/k/v/out are supported by the kernel", who);
  if (!std::isfinite(scale)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: scale must be finite", who);
  for (const void* ptr : {q, k, v, out, static_cast<const void*>(initial_state), static_cast<const void*>(final_state)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: tensors must be 16-byte aligned", who);
  return TOKMIX_OK;
}

}  // namespace gdn
}  // namespace tokmix

extern "C" int tokmix_gdn_prefill(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  const float* initial_state, void* out, float* final_state,
                                  const int32_t* cu_seqlens_dev, const int32_t* seq_order_dev, int num_seqs,
                                  int total_tokens, int heads_k, int heads_v, int head_dim_k, int head_dim_v,
                                  float scale, int io_dtype, const tokmix_gdn_stage1* gates, uint32_t* status,
                                  void* stream) {
  using namespace tokmix;
  using namespace tokmix::gdn;
  if (const int rc = validate_prefill_args("tokmix_gdn_prefill", q, k, v, g, beta, initial_state, out, final_state,
                                           num_seqs, total_tokens, heads_k, heads_v, head_dim_k, head_dim_v, scale,
                                           io_dtype, gates))
    return rc;
  if (cu_seqlens_dev == nullptr)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: null pointer argument");
  if (status == nullptr)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill: a device status word is required");
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
  p.num_seqs = num_seqs;
  p.total_tokens = total_tokens;
  if (stage1_gates(gates))
    p.gates = GateSource{gates->a, gates->b, gates->a_log, gates->dt_bias, gates->dtype == TOKMIX_DTYPE_BF16 ? 1 : 0};
  if (stage1_l2norm(gates)) {
    p.l2norm = 1;
    p.l2norm_eps = gates->l2norm_eps;
  }
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

// Device address of the current device's copy of g_scratch.  Set-up, once per device, with that
// device current: in host code the symbol is only a stand-in, the kernels need this address.
int scratch_base(int32_t** base) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(TOKMIX_ERR_DEVICE, "tokmix_gdn_prefill_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_base[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess)
      return fail(TOKMIX_ERR_DEVICE, "tokmix_gdn_prefill_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_base[dev] = static_cast<int32_t*>(ptr);
  }
  *base = g_base[dev];
  return TOKMIX_OK;
}

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
  // every check of the regular entry point that can fail runs before anything is enqueued, so a
  // rejected call leaves the shared array (and a call still running on it) untouched
  if (const int rc = gdn::validate_prefill_args("tokmix_gdn_prefill_noalloc", q, k, v, g, beta, initial_state, out,
                                                final_state, batch, batch * seqlen, heads_k, heads_v, head_dim_k,
                                                head_dim_v, scale, io_dtype))
    return rc;
  if (batch == 0) return TOKMIX_OK;
  if (const int rc = check_device()) return rc;
  int32_t* base = nullptr;
  if (const int rc = na::scratch_base(&base)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* st = status != nullptr ? status : reinterpret_cast<uint32_t*>(base);
  int32_t* offsets = base + 64;
  na::fill_offsets<<<(batch + 1 + 255) / 256, 256, 0, s>>>(offsets, batch, seqlen, status != nullptr ? nullptr : st);
  if (const int rc = check_launch("tokmix_gdn_prefill_noalloc")) return rc;
  return tokmix_gdn_prefill(q, k, v, g, beta, initial_state, out, final_state, offsets, nullptr, batch, batch * seqlen,
                            heads_k, heads_v, head_dim_k, head_dim_v, scale, io_dtype, nullptr, st, stream);
}

// Reads the library-owned status word of the current device that tokmix_gdn_prefill_noalloc
// uses when it is called with status == NULL (each such call clears it when it starts), with a
// synchronous copy; clear != 0 zeroes it afterwards.  Allocates nothing.
extern "C" int tokmix_gdn_noalloc_status(uint32_t* host_status, int clear) {
  using namespace tokmix;
  namespace na = tokmix::gdn::noalloc;
  if (host_status == nullptr) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_noalloc_status: null pointer");
  if (const int rc = check_device()) return rc;
  int32_t* base = nullptr;
  if (const int rc = na::scratch_base(&base)) return rc;
  cudaError_t e = cudaMemcpyFromSymbol(host_status, na::g_scratch, sizeof(uint32_t), 0, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear != 0) {
    const int32_t zero = 0;
    e = cudaMemcpyToSymbol(na::g_scratch, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess)
    return fail(TOKMIX_ERR_LAUNCH, "tokmix_gdn_noalloc_status: reading the status word failed: %s",
                cudaGetErrorString(e));
  return TOKMIX_OK;
}
