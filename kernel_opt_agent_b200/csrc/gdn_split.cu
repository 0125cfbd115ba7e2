// gdn_split.cu -- GDN prefill in two launches, for problems with few (sequence, value head)
// units, where one CTA per unit would leave most SMs idle and put a long per-chunk preparation
// path in front of every step of the state chain.
//
//   1. gdn_prep_kernel: every (chunk, value head) record, persistent CTAs (three per SM) taking
//      records in chunk-major order.  Decay sums, Q K^T / K K^T (tcgen05), the read-out of L, P
//      and e^G-scaled Q, the triangular solve, T and T diag(e^G), W = T diag(e^G) K (tcgen05).
//      Each of the chunk's MMA operands is staged in shared memory as its image in the
//      128-byte-swizzled layout the chain kernel feeds to the tensor core, and bulk-copied to one
//      record of kRecBytes in a workspace.
//   2. gdn_chain_kernel: one CTA per (sequence, value head).  A loader warp streams each chunk's
//      record (bulk copies) and its K, V tiles (TMA) into a two-stage ring; the state chain and
//      the output pass are those of gdn_prefill.cu without any preparation work.
// Results equal gdn_prefill.cu's bit for bit: the same operands and splits, and every TMEM
// accumulator receives its MMAs in the same order.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "gdn_common.cuh"
#include "gdn_segment.cuh"
#include "host_common.h"

namespace tokmix {
namespace gdn {
namespace split {

// ---- workspace record of one (chunk, value head)
constexpr int kRecT = 0;                      // T hi | lo, MN-major [s][t], 8 KB each
constexpr int kRecW = 16384;                  // -W hi | lo, [k][t], 16 KB each
constexpr int kRecQ = 49152;                  // scale e^G Q, K-major [t][k]: two 64-column boxes of 8 KB
constexpr int kRecP = 65536;                  // scale P, K-major [t][s], 8 KB
constexpr int kRecParams = 73728;             // ChunkParams
constexpr int kRecBytes = kRecParams + kParamsBytes;

// ---- preparation kernel
constexpr int kPrepThreads = 128;
constexpr int kPSlot = 0;                     // [K;Q]: two boxes of 128 rows x 128 B (K rows 0-63, Q 64-127)
constexpr int kPL = 32768;                    // L fp32 (row stride kLds); then T diag(e^G) hi | lo
constexpr int kPX = kPL + 64 * kLds * 4;      // X = (I + L)^-1 fp32
constexpr int kPParams = kPX + 64 * kLds * 4;
constexpr int kPSmem = kPParams + kParamsBytes;
constexpr int kPrepCtasPerSm = 3;
static_assert(kPL % 1024 == 0 && kPX % 16 == 0 && kPrepCtasPerSm * (kPSmem + 1024 + 64) <= 228 * 1024,
              "prep layout: three CTAs per SM");
// The record leaves shared memory by bulk copies, each tile staged as its exact image in a region
// that is dead by then: e^G Q in place in the Q rows; T hi | lo in the Q rows once that copy has
// read them; after T2, -W hi in L, -W lo in X and P in the K rows of box 0.
constexpr int kPQ0 = kPSlot + 8192, kPQ1 = kPSlot + 24576;  // the Q rows of boxes 0 and 1 (8 KB each)

// ---- chain kernel
constexpr int kChainThreads = 320;            // warps 0-7 passes, 8 loader, 9 MMA issuer
constexpr int kSK = 75776;                    // K: two boxes of 64 rows x 128 B (after the record)
constexpr int kSV = kSK + 16384;              // V: two boxes of 64 rows x 128 B
constexpr int kStageBytes = kSV + 16384;
constexpr int kCSmem = 2 * kStageBytes;
static_assert(kRecBytes <= kSK && kSK % 1024 == 0 && kStageBytes % 1024 == 0, "chain layout");
static_assert(kCSmem + 1024 + 256 <= 227 * 1024, "chain shared memory budget");

// Optional phase trace of the chain kernel (build with -DTOKMIX_GDN_TRACE): SM clock stamps of
// CTA 0 by event and chunk, read back with tokmix_gdn_split_trace_read().
#ifdef TOKMIX_GDN_TRACE
constexpr int kTrChunks = 64, kTrEvents = 16;
__device__ unsigned long long g_split_trace[kTrEvents * kTrChunks];
__device__ unsigned long long g_cta_end[1024];    // %globaltimer at the end of each CTA
__device__ unsigned long long g_cta_start[1024];  // %globaltimer at the start of each CTA
__device__ unsigned long long g_rec_start[2048];  // %globaltimer: overlapped launch, record rid begun
__device__ unsigned long long g_rec_end[2048];    // ... and published
__device__ unsigned long long g_chain_issue[64];  // ... chain CTA 0's loader: chunk c's copies issued
#define OVL_TRACE(arr, i, n)                                      \
  do {                                                            \
    if ((i) >= 0 && (i) < (n)) arr[(i)] = global_timer_ns();       \
  } while (0)
#define SPLIT_TRACE(ev, c)                                                                               \
  do {                                                                                                   \
    if (blockIdx.x == 0 && (c) < kTrChunks) g_split_trace[(ev) * kTrChunks + (c)] = clock64();          \
  } while (0)
#else
#define SPLIT_TRACE(ev, c) \
  do {                     \
  } while (0)
#define OVL_TRACE(arr, i, n) \
  do {                       \
  } while (0)
#endif
#ifdef TOKMIX_GDN_TRACE
// prep phases of the records of chunks [X0, X0 + 8) and value head Y prepared by the preparation
// launch (named barrier 1), by thread 0 (SM clock)
#ifndef TOKMIX_PREP_TRACE_Y
#define TOKMIX_PREP_TRACE_Y 0
#endif
#ifndef TOKMIX_PREP_TRACE_X0
#define TOKMIX_PREP_TRACE_X0 0
#endif
constexpr int kPrepTrCtas = 8, kPrepTrEvents = 16;
__device__ unsigned long long g_prep_trace[kPrepTrCtas * kPrepTrEvents];
#define PREP_TRACE(ev)                                                                         \
  do {                                                                                         \
    if (bar_id == 1 && h == TOKMIX_PREP_TRACE_Y && gc >= TOKMIX_PREP_TRACE_X0 &&                      \
        gc < TOKMIX_PREP_TRACE_X0 + kPrepTrCtas && tid == 0)                                           \
      g_prep_trace[(gc - TOKMIX_PREP_TRACE_X0) * kPrepTrEvents + (ev)] = clock64();               \
  } while (0)
#else
#define PREP_TRACE(ev) \
  do {                 \
  } while (0)
#endif
#ifdef TOKMIX_GDN_TRACE
#define CTA_END_TRACE()                                                                  \
  do {                                                                                   \
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_end[blockIdx.x] = global_timer_ns(); \
  } while (0)
#define CTA_START_TRACE()                                                                  \
  do {                                                                                     \
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_start[blockIdx.x] = global_timer_ns(); \
  } while (0)
#else
#define CTA_END_TRACE() \
  do {                  \
  } while (0)
#define CTA_START_TRACE() \
  do {                    \
  } while (0)
#endif

struct PrepParams {
  const float* g;
  const float* beta;
  const int32_t* cu_seqlens;
  const int32_t* chunk_base;  // [num_seqs + 1]: first global chunk of each sequence
  uint8_t* ws;
  int num_seqs, hk, hv;
  int total_tokens;
  float scale;
  uint32_t* status;
  GateSource gates;  // a == null: g and beta as given
  int l2norm;        // normalise the staged q and k rows before T1; the key head's first value
  float l2norm_eps;  //   head's record also writes the normalised keys to k_normed for the chains
  __nv_bfloat16* k_normed;
};

// A chain unit of the segmented schedule: `nchunks` chunks of sequence `seq` from its chunk
// `chunk0` on, for every value head.  kind:
//   kSegWhole  the whole sequence: initial state -> state_out[seq]; outputs to out
//   kSegFirst  its first segment: initial state -> seg_states[slot]; outputs to out
//   kSegLocal  a later segment from a zero state: real V; end state -> seg_states[slot]; outputs
//              (the segment's part that does not depend on its entry state) to out
//   kSegTrans  the same segment from the identity with V = 0: its end state (the segment's
//              transition matrix) -> seg_states[slot]; its outputs R (the entry state's share of
//              the outputs is R times the entry state transposed) to r_out
struct SegUnit {
  int32_t seq, chunk0, nchunks, kind_slot;  // kind in the low 2 bits, slot above
};
constexpr int kSegWhole = 0, kSegFirst = 1, kSegLocal = 2, kSegTrans = 3;

struct ChainParams {
  const float* state_in;
  float* state_out;
  float* checkpoints;  // [total_chunks, hv, 128, 128] or null: the state after each chunk
  __nv_bfloat16* out;
  const int32_t* cu_seqlens;
  const int32_t* chunk_base;
  const uint8_t* ws;
  int hk, hv;
  int total_tokens, total_chunks;
  uint32_t* status;
  // segmented schedule (units == null: unit u is (sequence u / hv, head u % hv), kind kSegWhole)
  const SegUnit* units;
  int num_units, num_slots, num_seqs;
  float* seg_states;      // [num_slots, hv, 128, 128]
  __nv_bfloat16* r_out;   // [total_tokens, hv, 128]
  // with flags (one cooperative launch) and normalised keys: the keys of chunk c are written by
  // the record of the key head's first value head, so the loader waits for that record too
  int wait_key_record;
};

// bulk copy global -> shared, completing on an mbarrier (one destination CTA)
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(sdst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// bulk copy shared -> global in the issuing thread's bulk group (both addresses 16-byte aligned,
// bytes a multiple of 16); bulk_commit closes the group, bulk_wait_read waits until every committed
// group has read its shared memory, bulk_wait until their global writes are done
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One record: the preparation of chunk gc of value head h by a group of 128 threads (group-local
// `tid`; the group's warp w must sit on TMEM lane quadrant w).  `smem` is the group's 1024-byte
// aligned region of kPSmem bytes, `tbase` its 64 TMEM columns, `bar_id` its named barrier;
// bar_in completes once per record (`in_parity`), bar_mma twice (parities 0, 1).  Returns false
// if a wait ran out.  The record (T, -W, e^G Q, P, params) is written to p.ws directly.
__device__ __forceinline__ bool prep_record(const CUtensorMap* map_q, const CUtensorMap* map_k, const PrepParams& p,
                                            int gc, int h, uint8_t* smem, uint64_t* bar_in, uint32_t in_parity,
                                            uint64_t* bar_mma, uint32_t tbase, int tid, int bar_id) {
  const int warp = tid >> 5, lane = tid & 31;
  PREP_TRACE(0);
  int lo = 0, hi = p.num_seqs;  // sequence of global chunk gc: chunk_base[lo] <= gc < chunk_base[lo + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.chunk_base[mid] <= gc) lo = mid; else hi = mid;
  }
  // token offsets and chunk bases are device data the host does not read: a chunk that falls
  // outside [0, total_tokens) sets TOKMIX_DEV_BAD_ARGS and reads no g / beta (its TMA loads stay
  // in bounds on their own: rows outside the tensor read as zero)
  const int seq = lo;
  const long long c_ll = static_cast<long long>(gc) - p.chunk_base[seq];
  const long long row_ll = p.cu_seqlens[seq] + c_ll * kC;
  const long long valid_ll = min(static_cast<long long>(kC), static_cast<long long>(p.cu_seqlens[seq + 1]) - row_ll);
  const bool bad = c_ll < 0 || row_ll < 0 || row_ll + max(valid_ll, 0ll) > p.total_tokens;
  if (bad && tid == 0) record_status(p.status, kDevBadArgs);
  const int n_valid = bad ? 0 : static_cast<int>(valid_ll);
  const int row0 = bad ? 0 : static_cast<int>(row_ll);
  const int kh = h % p.hk;
  ChunkParams& pc = *reinterpret_cast<ChunkParams*>(smem + kPParams);
  float* Ls = reinterpret_cast<float*>(smem + kPL);
  const PaddedRows X{reinterpret_cast<float*>(smem + kPX)};
  uint8_t* rec = p.ws + (static_cast<size_t>(gc) * p.hv + h) * kRecBytes;

  if (tid == 0) {
    mbar_arrive_expect_tx(bar_in, 32768);
    for (int bx = 0; bx < 2; ++bx) {
      tma_load_3d(smem + kPSlot + bx * 16384, map_k, bar_in, bx * 64, kh, row0);
      tma_load_3d(smem + kPSlot + bx * 16384 + 8192, map_q, bar_in, bx * 64, kh, row0);
    }
  }
  if (warp == 3) {
    const int t0 = 2 * lane, t1 = 2 * lane + 1;
    const size_t base = static_cast<size_t>(row0);
    float ga = 0.0f, gb = 0.0f, ba = 0.0f, bb = 0.0f;
    if (t0 < n_valid) load_gates(p.g, p.beta, p.gates, (base + t0) * p.hv + h, h, ga, ba);
    if (t1 < n_valid) load_gates(p.g, p.beta, p.gates, (base + t1) * p.hv + h, h, gb, bb);
    chunk_decay_params(pc, ga, gb, ba, bb, n_valid, lane);
  }
  named_sync(bar_id, 128);
  PREP_TRACE(1);
  // --- qk_l2norm: thread = row of the staged [K; Q] tile, normalised in place once it landed
  if (p.l2norm) {
    const bool landed = __all_sync(0xffffffffu, mbar_wait(bar_in, in_parity, p.status, kDevTimeoutTma));
    if (landed) {
      uint8_t* r0p = smem + kPSlot + tid * 128;
      l2norm_row_sw128(r0p, r0p + 16384, tid & 7, p.l2norm_eps);
      if (tid < n_valid && h < p.hk)  // rows 0-63 are keys; one value head per key head writes them
        copy_row_sw128(r0p, r0p + 16384, tid & 7, p.k_normed + (static_cast<size_t>(row0 + tid) * p.hk + kh) * kD);
      fence_async_smem();
    }
    if (!named_sync_and(bar_id, 128, landed)) return false;
  }
  // --- T1: [K;Q] K^T
  if (tid == 0 && mbar_wait(bar_in, in_parity, p.status, kDevTimeoutTma)) {
    tc_fence_after();
    const uint32_t id = make_idesc(128, 64, 1, 0, 0);
    const uint32_t slot = smem_u32(smem + kPSlot);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16_ss(tbase, kmaj_desc(slot, kk, 16384), kmaj_desc(slot, kk, 16384), id, kk > 0 ? 1u : 0u);
    umma_commit(bar_mma);
    PREP_TRACE(2);
  }
  // --- read-out: rows 0-63 (K K^T) -> L; the Q rows scaled in place to scale e^G Q, which a bulk
  //     copy stores.  Q K^T stays in TMEM columns 0-63 until P is formed at the end.
  bool ok = __all_sync(0xffffffffu, mbar_wait(bar_mma, 0, p.status, kDevTimeoutMma));
  PREP_TRACE(3);
  if (ok) {
    if (tid < 64) {
      tc_fence_after();
      uint32_t row[64];
      tmem_ld64(tmem_addr(tbase, warp * 32, 0), row);
      l_row(row, pc, tid, Ls);
    } else {
      const int t = tid - 64;
      scale_row_inplace(smem + kPQ0 + t * 128, kPQ1 - kPQ0, pc.eg[t] * p.scale);
    }
  }
  PREP_TRACE(12);
  fence_async_smem();  // the scaled Q rows -> the bulk copy
  tc_fence_before();
  ok = named_sync_and(bar_id, 128, ok);
  if (!ok) return false;
  if (tid == 0) {
    bulk_s2g(rec + kRecQ, smem + kPQ0, 8192);
    bulk_s2g(rec + kRecQ + 8192, smem + kPQ1, 8192);
    bulk_commit();
  }
  PREP_TRACE(4);
  // the solve's diagonal blocks on warps 0-1; meanwhile warps 2-3 (TMEM lanes 64-127) form their
  // row of P from Q K^T, kept in registers until the K rows are free after T2
  uint32_t prow[32];
  solve_inverse(Ls, X, tid, bar_id, 0, [&](int t) {
    tc_fence_after();
    uint32_t row[64];
    tmem_ld64(tmem_addr(tbase, warp * 32, 0), row);
    p_row_pack(row, pc, t - 64, p.scale, prow);
  });
  PREP_TRACE(5);
  if (tid == 0) bulk_wait_read();  // the Q rows are free for the T tiles
  named_sync(bar_id, 128);
  write_t_tiles(X, pc, tid, smem + kPQ0, smem + kPL, kPQ1 - kPQ0);  // T -> the Q rows, T diag(e^G) over the dead L
  fence_async_smem();
  named_sync(bar_id, 128);
  PREP_TRACE(6);
  // --- T2: W^T = K^T (TG_hi + TG_lo)^T into TMEM columns 64-127; the T tiles leave meanwhile
  if (tid == 0) {
    bulk_s2g(rec + kRecT, smem + kPQ0, 8192);
    bulk_s2g(rec + kRecT + 8192, smem + kPQ1, 8192);
    bulk_commit();
    tc_fence_after();
    const uint32_t id = make_idesc(128, 64, 1, 1, 1);
    const uint32_t kt = smem_u32(smem + kPSlot), tg = smem_u32(smem + kPL);
#pragma unroll
    for (int part = 0; part < 2; ++part)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(tbase + 64, make_sdesc_sw128(kt + kk * 2048, 16384, 1024),
                     make_sdesc_sw128(tg + part * 8192 + kk * 2048, 16384, 1024), id, (part > 0 || kk > 0) ? 1u : 0u);
    umma_commit(bar_mma);
    PREP_TRACE(7);
  }
  // --- -W hi | lo -> the dead L | X, P -> the dead K rows of box 0 (T2 has read K, TG, X)
  ok = __all_sync(0xffffffffu, mbar_wait(bar_mma, 1, p.status, kDevTimeoutMma));
  PREP_TRACE(8);
  if (ok) {
    tc_fence_after();
    uint32_t row[64];
    tmem_ld64(tmem_addr(tbase, warp * 32, 64), row);
    w_row(row, tid, smem + kPL, kPX - kPL);
    if (tid >= 64) store_row_sw128(smem + kPSlot, tid - 64, prow);
  }
  PREP_TRACE(10);
  fence_async_smem();
  tc_fence_before();
  ok = named_sync_and(bar_id, 128, ok);  // every TMEM read and staged tile of this record is done
  PREP_TRACE(11);
  if (ok && tid == 0) {
    bulk_s2g(rec + kRecW, smem + kPL, 16384);
    bulk_s2g(rec + kRecW + 16384, smem + kPX, 16384);
    bulk_s2g(rec + kRecP, smem + kPSlot, 8192);
    bulk_s2g(rec + kRecParams, smem + kPParams, kParamsBytes);
    bulk_commit();
  }
  PREP_TRACE(9);
  return ok;
}

// Persistent: CTA i prepares records i, i + gridDim.x, ... of the `records` = total chunks x heads_v
// records in chunk-major order (record r = chunk r / hv, value head r % hv, so the value heads of a
// key head, which load the same q and k rows, are prepared together).  Barriers, TMEM and the
// tensor maps are set up once per CTA.
__global__ void __launch_bounds__(kPrepThreads, kPrepCtasPerSm)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const PrepParams p, int records) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in, bar_mma;
  __shared__ uint32_t tmem_base_shared;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    cta_abort_flag() = 0u;
    mbar_init(&bar_in, 1);
    mbar_init(&bar_mma, 1);
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_shared, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_shared;
  uint32_t k = 0;
  for (int r = blockIdx.x; r < records; r += gridDim.x, ++k) {
    const int gc = r / p.hv, h = r - gc * p.hv;
    const bool ok = prep_record(&map_q, &map_k, p, gc, h, smem, &bar_in, k & 1, &bar_mma, tbase, tid, 1);
    // the record's bulk copies have read shared memory before the next record's loads and
    // parameter writes reuse it (their global writes complete on their own, before the launch ends)
    if (tid == 0) bulk_wait_read();
    named_sync(1, kPrepThreads);
    if (!ok) break;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

// Two-slot barrier helpers (event of chunk c in slot c & 1, phase (c >> 1) & 1)
__device__ __forceinline__ bool wait2(uint64_t* bars, int c, uint32_t* status, uint32_t code) {
  return mbar_wait(&bars[c & 1], (c >> 1) & 1, status, code);
}
__device__ __forceinline__ bool wait2_warp(uint64_t* bars, int c, uint32_t* status, uint32_t code) {
  return __all_sync(0xffffffffu, wait2(bars, c, status, code));
}

// Warp roles of a chain CTA.  Warps 0-7 are the pass warps: warp w and warp w + 4 share TMEM lane
// quadrant w (value rows 32(w & 3) .. +31) and take one half each of every pass's columns.  Warp 8
// (lane 0) loads, warp 9 (lane 0) issues every MMA: an issuing thread stalls for about as long as
// its MMAs take, so no pass warp issues.  The pass warps and the issuer warp meet twice per chunk
// on named barrier 1 (Delta pass done, state pass done).
constexpr int kPassThreads = 256;
constexpr int kSyncThreads = kPassThreads + 32;

// Every waiter of event c on a two-slot barrier waits before event c + 2 can complete (each
// producer of c + 2 causally follows each waiter of c), so a parity never goes two phases ahead.
struct ChainBarriers {
  uint64_t full[2];      // stage of chunk c loaded.                         waiters: issuer, pass warps, loader drain
  uint64_t tv_done[2];   // T V(c) complete.                                 waiter: issuer
  uint64_t x_ready[2];   // state terms(c) complete.                         waiters: pass warps
  uint64_t t3b_done[2];  // T3b(c) complete: S_hi, S_lo no longer read.      waiters: pass warps
  uint64_t s_new[2];     // T4(c) complete.                                  waiters: pass warps, loader
  uint64_t o_done[2];    // T5(c) (and so T3b(c)) complete.                  waiters: pass warps, loader
  uint64_t o_read[2];    // O(c) read out (one arrival per pass warp).       waiter: issuer
  uint64_t drain;
};

// TMEM columns of a chain CTA: the fp32 state S (the accumulator T4 adds to), its bf16 hi/lo
// copies (A operands of the state terms and T3b), X (T V, then the state terms: two 64-column
// partial sums of Delta), O (T3b + T5), and the bf16 Delta operands written by the Delta pass.
// The plain Delta (T5's A operand) lives in the first 32 S_lo columns: S_lo is dead from the end of
// the state terms (x_ready) until the state pass rewrites it after T5 has completed (o_done), and
// X is then free for T V(c+1) as soon as the Delta pass has read it.
constexpr uint32_t kColS = 0, kColShi = 128, kColSlo = 192, kColX = 256, kColO = 384;
constexpr uint32_t kColDhi = 448, kColDlo = 480;  // e^(G_C - G) Delta hi | lo (T4's A operand)
constexpr uint32_t kColDp = kColSlo;              // plain bf16 Delta, tokens 2j, 2j+1 in column j

// Barrier initialisation and TMEM allocation of a chain CTA (whole CTA); returns the TMEM base.
__device__ __forceinline__ uint32_t chain_setup(ChainBarriers& bars, uint32_t* tmem_base_shared) {
  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    uint64_t* all = reinterpret_cast<uint64_t*>(&bars);
    for (int i = 0; i < static_cast<int>(sizeof(ChainBarriers) / 8); ++i) mbar_init(&all[i], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&bars.o_read[i], kPassThreads / 32);
    fence_barrier_init();
  }
  if (warp_id() == 0) {
    tmem_alloc(tmem_base_shared, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *tmem_base_shared;
}

// The state chain of one (sequence, value head) unit on warps 0-9 (roles above), with `bars`
// initialised and 512 TMEM columns at `tbase`.  With `flags` non-null the loader waits (bounded)
// for flags[record] before it reads a record: the records are then being written by other CTAs
// of the same cooperative launch.
//
// Per chunk c (the critical path is marked *):
//   issuer  * state terms(c) once T V(c) is done; T3b(c) once O(c-1) is read out
//   pass    gamma pass: S(c) -> gamma_c S(c) and read-out of O(c-1), beside the state terms
//   pass    * Delta pass once x_ready(c)                                  -> barrier
//   issuer  * T4(c) -> s_new;  T5(c) -> o_done;  T V(c+1) (X is dead once the Delta pass read it)
//   pass    * state pass: S_hi of S(c+1) once s_new(c), t3b_done(c); S_lo once o_done(c) -> barrier
__device__ __forceinline__ void chain_unit(const CUtensorMap* map_k, const CUtensorMap* map_v, const ChainParams& p,
                                           uint8_t* smem, ChainBarriers& bars, uint32_t tbase, int unit,
                                           const uint32_t* flags) {
  const int warp = warp_id(), lane = lane_id();
  const int entry = unit / p.hv, h = unit - entry * p.hv;
  const int kh = h % p.hk;
  // Which tokens, start state and destinations this unit has.  The token offsets, chunk bases and
  // segment table are device data the host does not read: a unit whose entries are out of range
  // or inconsistent sets TOKMIX_DEV_BAD_ARGS and touches no memory.
  int seq = entry, chunk0 = 0, kind = kSegWhole, slot = 0;
  long long seg_chunks = -1;  // -1: the whole sequence
  if (p.units != nullptr) {
    const SegUnit su = p.units[entry];
    seq = su.seq;
    chunk0 = su.chunk0;
    seg_chunks = su.nchunks;
    kind = su.kind_slot & 3;
    slot = su.kind_slot >> 2;
  }
  bool bad = seq < 0 || seq >= p.num_seqs || chunk0 < 0 ||
             (kind != kSegWhole && (slot < 0 || slot >= p.num_slots || seg_chunks < 1));
  long long t_begin = 0, t_end = 0, gc_begin = 0;
  if (!bad) {
    const long long s_begin = p.cu_seqlens[seq], s_end = p.cu_seqlens[seq + 1];
    t_begin = s_begin + static_cast<long long>(chunk0) * kC;
    t_end = seg_chunks < 0 ? s_end : min(s_end, t_begin + seg_chunks * kC);
    gc_begin = static_cast<long long>(p.chunk_base[seq]) + chunk0;
    bad = s_begin < 0 || s_end < s_begin || s_end > p.total_tokens || t_begin > s_end ||
          (seg_chunks > 0 && t_end <= t_begin);
  }
  const long long n_chunks = t_end > t_begin ? (t_end - t_begin + kC - 1) / kC : 0;
  bad = bad || gc_begin < 0 || gc_begin + n_chunks > p.total_chunks;
  const int tok0 = bad ? 0 : static_cast<int>(t_begin);
  const int len = bad ? 0 : static_cast<int>(t_end - t_begin);
  const int N = len > 0 ? (len + kC - 1) / kC : 0;
  const int gc0 = bad ? 0 : static_cast<int>(gc_begin);
  if (bad && threadIdx.x == 0) record_status(p.status, kDevBadArgs);
  const bool zero_v = (kind == kSegTrans);
  // start state: the sequence's initial state (null: zero), zero, or the identity
  const float* s_in = (kind == kSegWhole || kind == kSegFirst) && p.state_in != nullptr
                          ? p.state_in + (static_cast<size_t>(seq) * p.hv + h) * kD * kD
                          : nullptr;
  const bool s_identity = (kind == kSegTrans);
  float* s_out = kind == kSegWhole ? p.state_out + (static_cast<size_t>(seq) * p.hv + h) * kD * kD
                                   : p.seg_states + (static_cast<size_t>(slot) * p.hv + h) * kD * kD;
  __nv_bfloat16* o_dst = zero_v ? p.r_out : p.out;
  float* const ckpt = kind == kSegWhole ? p.checkpoints : nullptr;
  auto stage = [&](int c) { return smem + (c & 1) * kStageBytes; };
  auto params_of = [&](int c) -> const ChunkParams& {
    return *reinterpret_cast<const ChunkParams*>(stage(c) + kRecParams);
  };

  if (N == 0) {
    if (warp < 4 && !bad) {
      const int v = threadIdx.x;
      for (int kk = 0; kk < kD; kk += 4) {
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s_in) val = *reinterpret_cast<const float4*>(s_in + v * kD + kk);
        *reinterpret_cast<float4*>(s_out + v * kD + kk) = val;
      }
    }
  } else if (warp == 8) {
    // ======================================================= loader: record + K + V per chunk
    if (lane == 0) {
      tma_prefetch_desc(map_k);
      tma_prefetch_desc(map_v);
      int issued = 0;
      for (int c = 0; c < N; ++c) {
        // the stage last held chunk c-2, whose MMAs (and so every read of its record, K and V)
        // have completed, and whose parameters the pass warps read before T4(c-2) was issued
        if (c >= 2 && !(wait2(bars.o_done, c - 2, p.status, kDevTimeoutPipe) &&
                        wait2(bars.s_new, c - 2, p.status, kDevTimeoutPipe)))
          break;
        SPLIT_TRACE(9, c);
        uint8_t* st = stage(c);
        uint64_t* bar = &bars.full[c & 1];
        const size_t ridx = static_cast<size_t>(gc0 + c) * p.hv + h;
        const uint8_t* rec = p.ws + ridx * kRecBytes;
        if (flags != nullptr && !wait_flag(flags + ridx, p.status)) break;
        if (flags != nullptr && p.wait_key_record && kh != h &&
            !wait_flag(flags + static_cast<size_t>(gc0 + c) * p.hv + kh, p.status))
          break;
        mbar_arrive_expect_tx(bar, kRecBytes + (zero_v ? 16384 : 32768));
        bulk_g2s(st, rec, kRecP, bar);  // T, W, e^G Q
        bulk_g2s(st + kRecP, rec + kRecP, kRecBytes - kRecP, bar);  // P, params
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_3d(st + kSK + bx * 8192, map_k, bar, bx * 64, kh, tok0 + c * kC);
          if (!zero_v) tma_load_3d(st + kSV + bx * 8192, map_v, bar, bx * 64, h, tok0 + c * kC);
        }
        if (blockIdx.x == 0) OVL_TRACE(g_chain_issue, c, 64);
        issued = c + 1;
      }
      for (int c = max(0, issued - 2); c < issued; ++c) mbar_drain(&bars.full[c & 1], (c >> 1) & 1);
    }
  } else if (warp == 9) {
    // ======================================================= MMA issuer (lane 0)
    const bool l0 = (lane == 0);
    // T V(c) = V^T [T_hi | T_lo]^T into the X region (accumulate 0)
    auto issue_tv = [&](int c) {
      const uint32_t st = smem_u32(stage(c));
      const uint32_t id_v = make_idesc(128, 128, 1, 1, 1);
      if (!zero_v) {  // with V = 0, T V is zero: the state terms start X instead
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16_ss(tbase + kColX, make_sdesc_sw128(st + kSV + kk * 2048, 8192, 1024),
                       make_sdesc_sw128(st + kRecT + kk * 2048, 8192, 1024), id_v, kk > 0 ? 1u : 0u);
      }
      umma_commit(&bars.tv_done[c & 1]);
      SPLIT_TRACE(12, c);
    };
    bool ok = true;
    if (l0) {
      ok = wait2(bars.full, 0, p.status, kDevTimeoutTma);
      if (ok) {
        tc_fence_after();
        issue_tv(0);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    ok = named_sync_and(1, kSyncThreads, ok);  // initial state and its hi/lo copies are in TMEM
    for (int c = 0; ok && c < N; ++c) {
      const uint32_t st = smem_u32(stage(c));
      if (l0) {
        // state terms(c): X += S_hi [-W_hi | -W_lo]^T (N = 128) + S_lo (-W_hi)^T (N = 64)
        ok = wait2(bars.tv_done, c, p.status, kDevTimeoutMma);
        SPLIT_TRACE(0, c);
        if (ok) {
          tc_fence_after();
          const uint32_t id128 = make_idesc(128, 128, 1, 0, 1), id64 = make_idesc(128, 64, 1, 0, 1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tbase + kColX, tbase + kColShi + 8 * kk, make_sdesc_sw128(st + kRecW + kk * 2048, 16384, 1024),
                         id128, (zero_v && kk == 0) ? 0u : 1u);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tbase + kColX, tbase + kColSlo + 8 * kk, make_sdesc_sw128(st + kRecW + kk * 2048, 16384, 1024),
                         id64, 1u);
          umma_commit(&bars.x_ready[c & 1]);
          SPLIT_TRACE(1, c);
          // T3b(c): O^T = S_hi (e^G Q)^T into the O region, once O(c-1) has been read out
          ok = (c == 0) || wait2(bars.o_read, c - 1, p.status, kDevTimeoutPipe);
        }
        if (ok) {
          tc_fence_after();
          const uint32_t id = make_idesc(128, 64, 1, 0, 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tbase + kColO, tbase + kColShi + 8 * kk, kmaj_desc(st + kRecQ, kk, 8192), id, kk > 0 ? 1u : 0u);
          umma_commit(&bars.t3b_done[c & 1]);
          SPLIT_TRACE(11, c);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      tc_fence_before();
      if (!named_sync_and(1, kSyncThreads, ok)) {  // Delta pass(c) done
        ok = false;
        break;
      }
      if (l0) {
        tc_fence_after();
        // T4(c): S^T += [Delta'_hi | Delta'_lo] [K; K] (gamma_c S(c) is in the S region)
        const uint32_t id_upd = make_idesc(128, 128, 1, 0, 1);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ts(tbase + kColS, tbase + kColDhi + 32 * part + 8 * kk,
                         make_sdesc_sw128(st + kSK + kk * 2048, 8192, 1024), id_upd, 1u);
        umma_commit(&bars.s_new[c & 1]);
        SPLIT_TRACE(4, c);
        // T5(c): O^T += Delta^T P^T (after T3b(c) and T4(c) in this thread's issue order)
        const uint32_t id = make_idesc(128, 64, 1, 0, 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16_ts(tbase + kColO, tbase + kColDp + 8 * kk, make_sdesc_sw128(st + kRecP + kk * 32, 16, 1024), id,
                       1u);
        umma_commit(&bars.o_done[c & 1]);
        SPLIT_TRACE(5, c);
        // T V(c+1): X was last read by the Delta pass (before the barrier above)
        if (c + 1 < N) {
          ok = wait2(bars.full, c + 1, p.status, kDevTimeoutTma);
          if (ok) {
            tc_fence_after();
            issue_tv(c + 1);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      tc_fence_before();
      if (!named_sync_and(1, kSyncThreads, ok)) {  // state pass(c) done
        ok = false;
        break;
      }
    }
    if (l0) {
      umma_commit(&bars.drain);
      mbar_drain(&bars.drain, 0);
    }
  } else {
    // ======================================================= pass warps 0-7 (lane = value row)
    const int q4 = warp & 3, hh = warp >> 2;
    const int v = q4 * 32 + lane;
    const uint32_t lb = tmem_addr(tbase, q4 * 32, 0);
    bool ok = true;
    {  // initial state S(0), key columns [64 hh, 64 hh + 64), and its hi/lo copies; gamma_0 is
       // applied by the gamma pass of chunk 0, so this does not wait for the first record
      uint32_t sv[64];
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s_in) val = *reinterpret_cast<const float4*>(s_in + v * kD + 64 * hh + j);
        sv[j] = __float_as_uint(val.x);
        sv[j + 1] = __float_as_uint(val.y);
        sv[j + 2] = __float_as_uint(val.z);
        sv[j + 3] = __float_as_uint(val.w);
      }
      if (s_identity) {  // the identity: row v has its 1 in key column v
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = (64 * hh + j == v) ? __float_as_uint(1.0f) : 0u;
      }
      store_split32<0>(lb + kColShi + 32 * hh, lb + kColSlo + 32 * hh, sv);
      store_split32<32>(lb + kColShi + 32 * hh + 16, lb + kColSlo + 32 * hh + 16, sv);
      tmem_st32(lb + kColS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_st32(lb + kColS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tmem_wait_st();
    }
    tc_fence_before();
    ok = named_sync_and(1, kSyncThreads, ok);

    // O(co) read-out, tokens [32 hh, 32 hh + 32) of the chunk: token pair (2i, 2i+1): the even
    // lane of a lane pair stores (O[2i][v], O[2i][v+1]), the odd lane (O[2i+1][v-1], O[2i+1][v]),
    // one 4-byte store each
    auto read_out = [&](int co) -> bool {
      if (!wait2_warp(bars.o_done, co, p.status, kDevTimeoutMma)) return false;
      tc_fence_after();
      if (threadIdx.x == 0) SPLIT_TRACE(10, co);
      uint32_t o[32];
      tmem_ld32(lb + kColO + 32 * hh, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.o_read[co & 1]);
      const int nv = min(kC, len - co * kC) - 32 * hh;
      const bool odd = (lane & 1) != 0;
      const size_t tstride = static_cast<size_t>(p.hv) * kD;
      uint32_t* dst = reinterpret_cast<uint32_t*>(o_dst + (static_cast<size_t>(tok0 + co * kC + 32 * hh) * p.hv + h) * kD +
                                                  (v & ~1)) + (odd ? tstride / 2 : 0);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float a = __uint_as_float(o[2 * i]), b = __uint_as_float(o[2 * i + 1]);
        const float other = __shfl_xor_sync(0xffffffffu, odd ? a : b, 1);
        const uint32_t packed = odd ? pack_bf16x2(other, b) : pack_bf16x2(a, other);
        if (2 * i + (odd ? 1 : 0) < nv) dst[i * tstride] = packed;
      }
      return true;
    };

    for (int c = 0; ok && c < N; ++c) {
      {
        // gamma pass: S(c) -> gamma_c S(c), the accumulator T4(c) adds to; then O(c-1).  Both run
        // beside the state-term MMAs, which read only S_hi, S_lo and write only X.
        ok = wait2_warp(bars.full, c, p.status, kDevTimeoutTma);
        if (threadIdx.x == 0) SPLIT_TRACE(7, c);
        if (ok) {
          const float gam = params_of(c).gamma_c;
          uint32_t sv[64];
          tmem_ld64(lb + kColS + 64 * hh, sv);
          if (ckpt != nullptr && c > 0) {  // S(c): the state after chunk c-1
            float* dst = ckpt + (static_cast<size_t>(gc0 + c - 1) * p.hv + h) * kD * kD + v * kD + 64 * hh;
#pragma unroll
            for (int j = 0; j < 64; j += 4)
              __stcs(reinterpret_cast<float4*>(dst + j), make_float4(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1]),
                                                                     __uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3])));
          }
#pragma unroll
          for (int j = 0; j < 64; ++j) sv[j] = __float_as_uint(__uint_as_float(sv[j]) * gam);
          tmem_st32(lb + kColS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_st32(lb + kColS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
          tmem_wait_st();
          if (c > 0) ok = read_out(c - 1);
        }
      }
      // --- Delta pass, tokens [32 hh, 32 hh + 32): Delta = X[t] + X[64 + t]; e^(G_C - G_t) Delta
      //     as hi/lo into the Delta columns, plain bf16 Delta into S_lo (read last by the state
      //     terms, complete at x_ready)
      const bool xr = ok && wait2_warp(bars.x_ready, c, p.status, kDevTimeoutMma);
      tc_fence_after();
      if (threadIdx.x == 0) SPLIT_TRACE(2, c);
      if (xr) {
        const ChunkParams& pc = params_of(c);
        uint32_t d[64];  // d[0..31] first partial sums, d[32..63] second
        tmem_ld32x2(lb + kColX + 32 * hh, lb + kColX + 64 + 32 * hh, d);
#pragma unroll
        for (int j = 0; j < 32; ++j) d[j] = __float_as_uint(__uint_as_float(d[j]) + __uint_as_float(d[32 + j]));
        uint32_t hi[16], lo[16], pk[16];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int t = 2 * j;
          const float4 e4 = *reinterpret_cast<const float4*>(&pc.egr[32 * hh + t]);
          split_pack(__uint_as_float(d[t]) * e4.x, __uint_as_float(d[t + 1]) * e4.y, hi[j], lo[j]);
          split_pack(__uint_as_float(d[t + 2]) * e4.z, __uint_as_float(d[t + 3]) * e4.w, hi[j + 1], lo[j + 1]);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(d[2 * j]), __uint_as_float(d[2 * j + 1]));
        tmem_st16(lb + kColDhi + 16 * hh, hi);
        tmem_st16(lb + kColDlo + 16 * hh, lo);
        tmem_st16(lb + kColDp + 16 * hh, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      if (!named_sync_and(1, kSyncThreads, xr)) {
        ok = false;
        break;
      }
      if (threadIdx.x == 0) SPLIT_TRACE(3, c);
      // --- state pass, key columns [64 hh, 64 hh + 64): hi/lo copies of S(c+1) -- hi after T3b(c)
      //     has read the old one, lo after T5(c) has read the plain Delta there -- or the final
      //     state after the last chunk
      const bool last = (c == N - 1);
      bool sr = wait2_warp(bars.s_new, c, p.status, kDevTimeoutMma) &&
                wait2_warp(bars.t3b_done, c, p.status, kDevTimeoutMma);
      tc_fence_after();
      if (threadIdx.x == 0) SPLIT_TRACE(6, c);
      if (sr) {
        uint32_t sv[64];
        tmem_ld64(lb + kColS + 64 * hh, sv);
        if (last) {
          float* dst = s_out + v * kD + 64 * hh;
          float* ck = ckpt != nullptr ? ckpt + (static_cast<size_t>(gc0 + c) * p.hv + h) * kD * kD + v * kD + 64 * hh
                                      : nullptr;
#pragma unroll
          for (int j = 0; j < 64; j += 4) {
            const float4 val = make_float4(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1]),
                                           __uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3]));
            *reinterpret_cast<float4*>(dst + j) = val;
            if (ck != nullptr) __stcs(reinterpret_cast<float4*>(ck + j), val);
          }
        } else {
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) split_pack(__uint_as_float(sv[2 * j]), __uint_as_float(sv[2 * j + 1]), hi[j], lo[j]);
          tmem_st32(lb + kColShi + 32 * hh, hi);
          sr = wait2_warp(bars.o_done, c, p.status, kDevTimeoutMma);
          tc_fence_after();
          if (sr) tmem_st32(lb + kColSlo + 32 * hh, lo);
          tmem_wait_st();
        }
      }
      tc_fence_before();
      if (!named_sync_and(1, kSyncThreads, sr)) {
        ok = false;
        break;
      }
      if (threadIdx.x == 0) SPLIT_TRACE(8, c);
    }
    if (ok) read_out(N - 1);
  }
}

__global__ void __launch_bounds__(kChainThreads, 1)
    gdn_chain_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                     const ChainParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ ChainBarriers bars;
  __shared__ uint32_t tmem_base_shared;
  const uint32_t tbase = chain_setup(bars, &tmem_base_shared);
  chain_unit(&map_k, &map_v, p, smem, bars, tbase, blockIdx.x, nullptr);
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---- one cooperative launch: chain CTAs and preparation CTAs side by side
constexpr int kOverlapThreads = 384;
constexpr int kPSmemA = (kPSmem + 1023) / 1024 * 1024;  // one preparation group's region
constexpr int kOSmem = kCSmem > 3 * kPSmemA ? kCSmem : 3 * kPSmemA;
static_assert(kOSmem + 1024 + 512 <= 227 * 1024, "overlap shared memory budget");

struct OverlapParams {
  const int32_t* record_order;  // [records]: record index (gc * heads_v + h) in chunk-major order
  uint32_t* flags;              // [records]: zero at launch; 1 once the record has been written
  int units;                    // CTAs [0, units) run the chain of one unit each
  int records;
};

// CTAs [0, units): the chain kernel's work for one unit (warps 0-8), whose loader waits for each
// record's flag.  The other CTAs: three preparation groups of 128 threads each, every group
// working through the records in chunk-major order (so the chains' first chunks come first) and
// publishing each finished record with a release store of its flag.  A cooperative launch keeps
// every CTA resident, so the chain CTAs' (bounded) waits are on CTAs that are running.
__global__ void __launch_bounds__(kOverlapThreads, 1)
    gdn_overlap_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_kc,
                       const PrepParams pp, const ChainParams cp, const OverlapParams op) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ ChainBarriers bars;
  __shared__ uint64_t pbar[3][2];
  __shared__ uint32_t tmem_base_shared;
  const int warp = warp_id();
  CTA_START_TRACE();
  if (static_cast<int>(blockIdx.x) < op.units) {
    const uint32_t tbase = chain_setup(bars, &tmem_base_shared);
    if (warp < kChainThreads / 32) chain_unit(&map_kc, &map_v, cp, smem, bars, tbase, blockIdx.x, op.flags);
    tc_fence_before();
    __syncthreads();
    CTA_END_TRACE();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tbase, 512);
    }
    return;
  }
  const int grp = threadIdx.x >> 7, tid = threadIdx.x & 127;
  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    for (int g = 0; g < 3; ++g) {
      mbar_init(&pbar[g][0], 1);
      mbar_init(&pbar[g][1], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_shared, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_shared + 128 * grp;
  // Slot (group, CTA) takes records grp * nprep + cta, + stride, ...: the first records -- the
  // chains' first chunk -- land one per SM, on groups 0; all groups start at once.
  const int nprep = gridDim.x - op.units;
  const int stride = nprep * 3;
  const int first = grp * nprep + (blockIdx.x - op.units);
  bool ok = true;
  uint32_t k = 0;
  for (int r = first; ok && r < op.records; r += stride, ++k) {
    const int rid = op.record_order[r];
    if (rid < 0 || rid >= op.records) {  // device data the host does not read
      if (tid == 0) record_status(pp.status, kDevBadArgs);
      continue;
    }
    const int gc = rid / pp.hv, h = rid - gc * pp.hv;
    if (tid == 0) OVL_TRACE(g_rec_start, rid, 2048);
    ok = prep_record(&map_q, &map_k, pp, gc, h, smem + grp * kPSmemA, &pbar[grp][0], k & 1, &pbar[grp][1], tbase, tid,
                     1 + grp);
    if (tid == 0) {
      // the record's bulk copies are written out (and have read the group's shared memory, which
      // the next record's loads overwrite); the direct stores of k_normed precede prep_record's
      // final group barrier
      bulk_wait();
      if (ok) {
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(op.flags + rid), "r"(1u) : "memory");
        OVL_TRACE(g_rec_end, rid, 2048);
      }
    }
    named_sync(1 + grp, 128);  // no thread writes the next record's parameters before the copies read them
  }
  tc_fence_before();
  __syncthreads();
  CTA_END_TRACE();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base_shared, 512);
  }
}

}  // namespace split
}  // namespace gdn
}  // namespace tokmix

#ifdef TOKMIX_GDN_TRACE
extern "C" int tokmix_gdn_split_cta_end_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn::split;
  const int count = n < 1024 ? n : 1024;
  return cudaMemcpyFromSymbol(host, g_cta_end, sizeof(unsigned long long) * count) == cudaSuccess ? count : -1;
}
extern "C" int tokmix_gdn_split_cta_start_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn::split;
  const int count = n < 1024 ? n : 1024;
  return cudaMemcpyFromSymbol(host, g_cta_start, sizeof(unsigned long long) * count) == cudaSuccess ? count : -1;
}
extern "C" int tokmix_gdn_overlap_trace_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn::split;
  if (n < 2048 * 2 + 64) return -1;
  if (cudaMemcpyFromSymbol(host, g_rec_start, sizeof(unsigned long long) * 2048) != cudaSuccess ||
      cudaMemcpyFromSymbol(host + 2048, g_rec_end, sizeof(unsigned long long) * 2048) != cudaSuccess ||
      cudaMemcpyFromSymbol(host + 4096, g_chain_issue, sizeof(unsigned long long) * 64) != cudaSuccess)
    return -1;
  return 2048 * 2 + 64;
}
extern "C" int tokmix_gdn_prep_trace_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn::split;
  const int count = n < kPrepTrCtas * kPrepTrEvents ? n : kPrepTrCtas * kPrepTrEvents;
  return cudaMemcpyFromSymbol(host, g_prep_trace, sizeof(unsigned long long) * count) == cudaSuccess ? count : -1;
}
extern "C" int tokmix_gdn_split_trace_read(unsigned long long* host, int n) {
  using namespace tokmix::gdn::split;
  const int count = n < kTrEvents * kTrChunks ? n : kTrEvents * kTrChunks;
  return cudaMemcpyFromSymbol(host, g_split_trace, sizeof(unsigned long long) * count) == cudaSuccess ? count : -1;
}
#endif

namespace tokmix {
namespace gdn {
namespace split {

static void set_l2norm(PrepParams& pp, const tokmix_gdn_stage1* s1) {
  if (!stage1_l2norm(s1)) return;
  pp.l2norm = 1;
  pp.l2norm_eps = s1->l2norm_eps;
  pp.k_normed = static_cast<__nv_bfloat16*>(s1->k_normed);
}

static GateSource gate_source(const tokmix_gdn_stage1* gates) {
  if (!stage1_gates(gates)) return GateSource{};
  return GateSource{gates->a, gates->b, gates->a_log, gates->dt_bias, gates->dtype == TOKMIX_DTYPE_BF16 ? 1 : 0};
}

// TMA maps over q, k [tokens, heads_k, 128] and v [tokens, heads_v, 128] (bf16); boxes of 64
// columns x 1 head x 64 tokens, 128-byte swizzle.
static bool encode_qkv_maps(const void* q, const void* k, const void* v, int total_tokens, int heads_k, int heads_v,
                            CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv) {
  const uint64_t rows = static_cast<uint64_t>(total_tokens > 0 ? total_tokens : 1);
  uint64_t dims_k[3] = {kD, static_cast<uint64_t>(heads_k), rows};
  uint64_t strides_k[2] = {kD * 2, static_cast<uint64_t>(heads_k) * kD * 2};
  uint64_t dims_v[3] = {kD, static_cast<uint64_t>(heads_v), rows};
  uint64_t strides_v[2] = {kD * 2, static_cast<uint64_t>(heads_v) * kD * 2};
  uint32_t box[3] = {64, 1, 64};
  return encode_tiled(mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims_k, strides_k, box, CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_tiled(mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims_k, strides_k, box, CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_tiled(mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims_v, strides_v, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace split
}  // namespace gdn
}  // namespace tokmix

// records of kRecBytes, then one uint32 ready flag per record (used by the overlapped launch)
extern "C" long long tokmix_gdn_split_workspace_bytes(int total_chunks, int heads_v) {
  if (total_chunks < 0 || heads_v < 0) return -1;
  const long long records = static_cast<long long>(total_chunks) * heads_v;
  return records * tokmix::gdn::split::kRecBytes + ((records * 4 + 255) / 256) * 256;
}

extern "C" int tokmix_gdn_prefill_split(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, const float* initial_state, void* out, float* final_state,
                                        float* checkpoints, const int32_t* cu_seqlens_dev, const int32_t* chunk_base_dev,
                                        const int32_t* record_order_dev, int num_seqs, int total_tokens,
                                        int total_chunks, int heads_k, int heads_v, int head_dim_k,
                                        int head_dim_v, float scale, int io_dtype,
                                        const tokmix_gdn_stage1* gates, void* workspace,
                                        long long workspace_bytes, uint32_t* status, void* stream) {
  using namespace tokmix;
  using namespace tokmix::gdn;
  using namespace tokmix::gdn::split;
  if (num_seqs < 0 || total_tokens < 0 || total_chunks < 0 || heads_k <= 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_split: negative or zero size");
  if (num_seqs == 0) return TOKMIX_OK;
  if (!q || !k || !v || !out || !final_state || !cu_seqlens_dev || !chunk_base_dev || !status ||
      (!stage1_gates(gates) && (!g || !beta)))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_split: null pointer argument");
  if (const int rc = check_stage1("tokmix_gdn_prefill_split", gates, true)) return rc;
  if (heads_v % heads_k != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT,
                "tokmix_gdn_prefill_split: heads_v (%d) must be a multiple of heads_k (%d)", heads_v, heads_k);
  if (head_dim_k != kD || head_dim_v != kD)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill_split: head dims must be 128 (got %d, %d)", head_dim_k,
                head_dim_v);
  if (io_dtype != TOKMIX_DTYPE_BF16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill_split: only bf16 q/k/v/out are supported by the kernel");
  if (!std::isfinite(scale)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_split: scale must be finite");
  const long long need = tokmix_gdn_split_workspace_bytes(total_chunks, heads_v);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_split: workspace of %lld bytes needed (got %lld)", need,
                workspace_bytes);
  for (const void* ptr : {q, k, v, static_cast<const void*>(out), static_cast<const void*>(initial_state),
                          static_cast<const void*>(final_state),
                          static_cast<const void*>(checkpoints), static_cast<const void*>(workspace)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_split: tensors must be 16-byte aligned");
  if (const int rc = check_device()) return rc;
  const long long units = static_cast<long long>(num_seqs) * heads_v;
  if (units > 0x7FFFFFFFll)
    return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_gdn_prefill_split: problem too large");

  CUtensorMap mq, mk, mv;
  if (!encode_qkv_maps(q, k, v, total_tokens, heads_k, heads_v, &mq, &mk, &mv)) return TOKMIX_ERR_INVALID_ARGUMENT;
  CUtensorMap mkc = mk;  // the chains' keys: the normalised copy when the preparation normalises
  if (stage1_l2norm(gates) && !encode_qkv_maps(q, gates->k_normed, v, total_tokens, heads_k, heads_v, &mq, &mkc, &mv))
    return TOKMIX_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PrepParams pp{};
  pp.g = g;
  pp.beta = beta;
  pp.cu_seqlens = cu_seqlens_dev;
  pp.chunk_base = chunk_base_dev;
  pp.ws = static_cast<uint8_t*>(workspace);
  pp.num_seqs = num_seqs;
  pp.total_tokens = total_tokens;
  pp.hk = heads_k;
  pp.hv = heads_v;
  pp.scale = scale;
  pp.status = status;
  pp.gates = gate_source(gates);
  set_l2norm(pp, gates);
  ChainParams cp{};
  cp.state_in = initial_state;
  cp.state_out = final_state;
  cp.checkpoints = checkpoints;
  cp.out = static_cast<__nv_bfloat16*>(out);
  cp.cu_seqlens = cu_seqlens_dev;
  cp.chunk_base = chunk_base_dev;
  cp.ws = static_cast<const uint8_t*>(workspace);
  cp.hk = heads_k;
  cp.hv = heads_v;
  cp.total_tokens = total_tokens;
  cp.total_chunks = total_chunks;
  cp.num_seqs = num_seqs;  // units == null: one whole-sequence unit per (sequence, head)
  cp.wait_key_record = stage1_l2norm(gates) ? 1 : 0;
  cp.status = status;
  const long long records = static_cast<long long>(total_chunks) * heads_v;
  // --- one cooperative launch when the chains leave SMs free for the preparation CTAs
  if (record_order_dev != nullptr && records > 0) {
    const int sms = device_sm_count();
    const int smem = kOSmem + 1024;
    int per_sm = 0;
    if (units + 8 <= sms && ensure_smem_attr(reinterpret_cast<const void*>(&gdn_overlap_kernel), smem) &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gdn_overlap_kernel, kOverlapThreads, smem) ==
            cudaSuccess &&
        per_sm >= 1) {
      OverlapParams op{};
      op.record_order = record_order_dev;
      op.flags = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + records * kRecBytes);
      op.units = static_cast<int>(units);
      op.records = static_cast<int>(records);
      if (cudaMemsetAsync(op.flags, 0, static_cast<size_t>(records) * 4, s) != cudaSuccess)
        return check_launch("tokmix_gdn_prefill_split: clearing the record flags");
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(static_cast<unsigned>(sms));
      cfg.blockDim = dim3(kOverlapThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, gdn_overlap_kernel, mq, mk, mv, mkc, pp, cp, op) == cudaSuccess)
        return check_launch("tokmix_gdn_prefill_split (overlapped)");
      cudaGetLastError();  // not launchable cooperatively here: two launches instead
    } else {
      cudaGetLastError();
    }
  }
  if (total_chunks > 0) {
    const int smem = kPSmem + 1024;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&gdn_prep_kernel), smem))
      return check_launch("tokmix_gdn_prefill_split: cudaFuncSetAttribute (prep)");
    const int records = total_chunks * heads_v;
    const int grid = std::min(records, kPrepCtasPerSm * std::max(1, device_sm_count()));
    gdn_prep_kernel<<<grid, kPrepThreads, smem, s>>>(mq, mk, pp, records);
    if (const int rc = check_launch("tokmix_gdn_prefill_split (prep)")) return rc;
  }
  const int smem = kCSmem + 1024;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(&gdn_chain_kernel), smem))
    return check_launch("tokmix_gdn_prefill_split: cudaFuncSetAttribute (chain)");
  gdn_chain_kernel<<<static_cast<unsigned>(units), kChainThreads, smem, s>>>(mkc, mv, cp);
  return check_launch("tokmix_gdn_prefill_split (chain)");
}

// ---------------------------------------------------------------------------------------------
// Segmented schedule: a long sequence's chunks are cut into segments that run side by side (see
// gdn_segment.cuh for the maths).  Host side: the plan (chain units, combine items, correction
// tiles), the workspace layout, and the entry point that launches preparation, chains, combine
// and correction in order on one stream.
namespace tokmix {
namespace gdn {
namespace segment {

struct Plan {
  std::vector<split::SegUnit> units;
  std::vector<CombineItem> combine;
  std::vector<CorrItem> corr;
  int num_slots = 0, num_eslots = 0;
  long long off_r = 0, off_states = 0, off_e = 0, off_units = 0, off_combine = 0, off_corr = 0, total = 0;
};

static long long round256(long long x) { return (x + 255) / 256 * 256; }

// Builds the plan from the host copy of the token offsets; returns false (error set) on
// inconsistent arguments.  Sequences of more than max_seg chunks are cut into the fewest
// near-equal segments of at most max_seg chunks.
static bool make_plan(const int32_t* cu, int num_seqs, int total_tokens, int total_chunks, int hv, int max_seg,
                      Plan& plan) {
  if (cu == nullptr || num_seqs < 0 || max_seg < 1) {
    fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_segmented: bad host offsets or max_segment_chunks");
    return false;
  }
  long long chunks = 0;
  for (int n = 0; n < num_seqs; ++n) {
    if (cu[n] < 0 || cu[n + 1] < cu[n]) {
      fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_prefill_segmented: host offsets must be non-decreasing from 0");
      return false;
    }
    chunks += (cu[n + 1] - cu[n] + kC - 1) / kC;
  }
  if (cu[0] != 0 || cu[num_seqs] != total_tokens || chunks != total_chunks) {
    fail(TOKMIX_ERR_INVALID_ARGUMENT,
         "tokmix_gdn_prefill_segmented: host offsets disagree with total_tokens / total_chunks");
    return false;
  }
  for (int n = 0; n < num_seqs; ++n) {
    const int len = cu[n + 1] - cu[n];
    const int nch = (len + kC - 1) / kC;
    if (nch <= max_seg) {
      plan.units.push_back({n, 0, -1, split::kSegWhole});
      continue;
    }
    const int nseg = (nch + max_seg - 1) / max_seg;
    const int base = nch / nseg, extra = nch % nseg;
    const int slot_base = plan.num_slots, e_base = plan.num_eslots;
    plan.num_slots += 2 * nseg - 1;
    plan.num_eslots += nseg - 1;
    int c0 = 0;
    for (int j = 0; j < nseg; ++j) {
      const int sz = base + (j < extra ? 1 : 0);
      if (j == 0) {
        plan.units.push_back({n, 0, sz, split::kSegFirst | (slot_base << 2)});
      } else {
        plan.units.push_back({n, c0, sz, split::kSegLocal | ((slot_base + 2 * j - 1) << 2)});
        plan.units.push_back({n, c0, sz, split::kSegTrans | ((slot_base + 2 * j) << 2)});
        const int t_begin = cu[n] + c0 * kC, t_end = std::min(cu[n + 1], cu[n] + (c0 + sz) * kC);
        for (int t = t_begin; t < t_end; t += 128)
          plan.corr.push_back({t, std::min(128, t_end - t), e_base + j - 1, 0});
      }
      c0 += sz;
    }
    plan.combine.push_back({n, nseg, slot_base, e_base});
  }
  // longest chains first
  std::stable_sort(plan.units.begin(), plan.units.end(), [&](const split::SegUnit& a, const split::SegUnit& b) {
    auto len = [&](const split::SegUnit& u) { return u.nchunks >= 0 ? u.nchunks : (cu[u.seq + 1] - cu[u.seq] + kC - 1) / kC; };
    return len(a) > len(b);
  });
  const long long records = static_cast<long long>(total_chunks) * hv;
  plan.off_r = round256(records * split::kRecBytes);
  plan.off_states = plan.off_r + round256(static_cast<long long>(total_tokens) * hv * kD * 2);
  plan.off_e = plan.off_states + round256(static_cast<long long>(plan.num_slots) * hv * kD * kD * 4);
  plan.off_units = plan.off_e + round256(static_cast<long long>(plan.num_eslots) * hv * kD * kD * 2);
  plan.off_combine = plan.off_units + round256(static_cast<long long>(plan.units.size()) * sizeof(split::SegUnit));
  plan.off_corr = plan.off_combine + round256(static_cast<long long>(plan.combine.size()) * sizeof(CombineItem));
  plan.total = plan.off_corr + round256(static_cast<long long>(plan.corr.size()) * sizeof(CorrItem));
  return true;
}

// The plan's tables as they lie in device memory: units, combine items, correction tiles, each
// section starting on a 256-byte boundary (the last plan.total - plan.off_units bytes of the
// workspace, or a separate device copy).
static void write_tables(const Plan& plan, uint8_t* dst) {
  std::memset(dst, 0, static_cast<size_t>(plan.total - plan.off_units));
  std::memcpy(dst, plan.units.data(), plan.units.size() * sizeof(split::SegUnit));
  std::memcpy(dst + (plan.off_combine - plan.off_units), plan.combine.data(), plan.combine.size() * sizeof(CombineItem));
  std::memcpy(dst + (plan.off_corr - plan.off_units), plan.corr.data(), plan.corr.size() * sizeof(CorrItem));
}

}  // namespace segment
}  // namespace gdn
}  // namespace tokmix

extern "C" long long tokmix_gdn_segmented_workspace_bytes(const int32_t* cu_seqlens_host, int num_seqs, int heads_v,
                                                          int max_segment_chunks) {
  using namespace tokmix::gdn;
  if (cu_seqlens_host == nullptr || num_seqs < 0 || heads_v <= 0 || max_segment_chunks < 1) return -1;
  long long chunks = 0;
  for (int n = 0; n < num_seqs; ++n) {
    if (cu_seqlens_host[n + 1] < cu_seqlens_host[n]) return -1;
    chunks += (cu_seqlens_host[n + 1] - cu_seqlens_host[n] + kC - 1) / kC;
  }
  if (chunks > 0x7FFFFFFFll) return -1;
  segment::Plan plan;
  if (!segment::make_plan(cu_seqlens_host, num_seqs, cu_seqlens_host[num_seqs], static_cast<int>(chunks), heads_v,
                          max_segment_chunks, plan))
    return -1;
  return plan.total;
}

// Size of the plan tables, and the tables themselves written to host memory (for a caller that
// keeps a device copy and passes it as plan_dev).
extern "C" long long tokmix_gdn_segmented_plan_bytes(const int32_t* cu_seqlens_host, int num_seqs, int heads_v,
                                                     int max_segment_chunks) {
  using namespace tokmix::gdn;
  const long long ws = tokmix_gdn_segmented_workspace_bytes(cu_seqlens_host, num_seqs, heads_v, max_segment_chunks);
  if (ws < 0) return -1;
  long long chunks = 0;
  for (int n = 0; n < num_seqs; ++n) chunks += (cu_seqlens_host[n + 1] - cu_seqlens_host[n] + kC - 1) / kC;
  segment::Plan plan;
  segment::make_plan(cu_seqlens_host, num_seqs, cu_seqlens_host[num_seqs], static_cast<int>(chunks), heads_v,
                     max_segment_chunks, plan);
  return plan.total - plan.off_units;
}

extern "C" int tokmix_gdn_segmented_plan(const int32_t* cu_seqlens_host, int num_seqs, int heads_v,
                                         int max_segment_chunks, void* plan_host, long long plan_bytes) {
  using namespace tokmix;
  using namespace tokmix::gdn;
  const long long need = tokmix_gdn_segmented_plan_bytes(cu_seqlens_host, num_seqs, heads_v, max_segment_chunks);
  if (need < 0) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_segmented_plan: inconsistent arguments");
  if (plan_host == nullptr || plan_bytes < need)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_gdn_segmented_plan: %lld bytes needed (got %lld)", need, plan_bytes);
  long long chunks = 0;
  for (int n = 0; n < num_seqs; ++n) chunks += (cu_seqlens_host[n + 1] - cu_seqlens_host[n] + kC - 1) / kC;
  segment::Plan plan;
  segment::make_plan(cu_seqlens_host, num_seqs, cu_seqlens_host[num_seqs], static_cast<int>(chunks), heads_v,
                     max_segment_chunks, plan);
  segment::write_tables(plan, static_cast<uint8_t*>(plan_host));
  return TOKMIX_OK;
}

extern "C" int tokmix_gdn_prefill_segmented(const void* q, const void* k, const void* v, const float* g,
                                            const float* beta, const float* initial_state, void* out,
                                            float* final_state, const int32_t* cu_seqlens_dev,
                                            const int32_t* chunk_base_dev, const int32_t* cu_seqlens_host,
                                            int num_seqs, int total_tokens, int total_chunks, int heads_k, int heads_v,
                                            int head_dim_k, int head_dim_v, float scale, int io_dtype,
                                            const tokmix_gdn_stage1* gates, int max_segment_chunks,
                                            const void* plan_dev, void* workspace, long long workspace_bytes,
                                            uint32_t* status, void* stream) {
  using namespace tokmix;
  using namespace tokmix::gdn;
  using namespace tokmix::gdn::split;
  const char* who = "tokmix_gdn_prefill_segmented";
  if (num_seqs < 0 || total_tokens < 0 || total_chunks < 0 || heads_k <= 0 || heads_v <= 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: negative or zero size", who);
  if (num_seqs == 0) return TOKMIX_OK;
  if (!q || !k || !v || !out || !final_state || !cu_seqlens_dev || !chunk_base_dev || !status ||
      (!stage1_gates(gates) && (!g || !beta)))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: null pointer argument", who);
  if (const int rc = check_stage1(who, gates, true)) return rc;
  if (heads_v % heads_k != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: heads_v (%d) must be a multiple of heads_k (%d)", who, heads_v, heads_k);
  if (head_dim_k != kD || head_dim_v != kD)
    return fail(TOKMIX_ERR_UNSUPPORTED, "%s: head dims must be 128 (got %d, %d)", who, head_dim_k, head_dim_v);
  if (io_dtype != TOKMIX_DTYPE_BF16)
    return fail(TOKMIX_ERR_UNSUPPORTED, "%s: only bf16 q/k/v/out are supported by the kernel", who);
  if (!std::isfinite(scale)) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: scale must be finite", who);
  for (const void* ptr : {q, k, v, static_cast<const void*>(out), static_cast<const void*>(initial_state),
                          static_cast<const void*>(final_state), static_cast<const void*>(workspace), plan_dev})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: tensors must be 16-byte aligned", who);
  segment::Plan plan;
  if (!segment::make_plan(cu_seqlens_host, num_seqs, total_tokens, total_chunks, heads_v, max_segment_chunks, plan))
    return TOKMIX_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < plan.total)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "%s: workspace of %lld bytes needed (got %lld)", who, plan.total,
                workspace_bytes);
  if (static_cast<long long>(plan.units.size()) * heads_v > 0x7FFFFFFFll ||
      static_cast<long long>(plan.corr.size()) > 0x7FFFFFFFll || plan.num_slots > (1 << 28))
    return fail(TOKMIX_ERR_UNSUPPORTED, "%s: problem too large", who);
  if (const int rc = check_device()) return rc;

  CUtensorMap mq, mk, mv;
  if (!encode_qkv_maps(q, k, v, total_tokens, heads_k, heads_v, &mq, &mk, &mv)) return TOKMIX_ERR_INVALID_ARGUMENT;
  CUtensorMap mkc = mk;  // the chains' keys: the normalised copy when the preparation normalises
  if (stage1_l2norm(gates) && !encode_qkv_maps(q, gates->k_normed, v, total_tokens, heads_k, heads_v, &mq, &mkc, &mv))
    return TOKMIX_ERR_INVALID_ARGUMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* r_out = reinterpret_cast<__nv_bfloat16*>(ws + plan.off_r);
  auto* seg_states = reinterpret_cast<float*>(ws + plan.off_states);
  auto* e_bf16 = reinterpret_cast<__nv_bfloat16*>(ws + plan.off_e);
  // the plan's tables: the caller's device copy, or the workspace's last bytes (uploaded below)
  const uint8_t* tables = plan_dev != nullptr ? static_cast<const uint8_t*>(plan_dev) : ws + plan.off_units;
  auto* units_dev = reinterpret_cast<const SegUnit*>(tables);
  auto* combine_dev = reinterpret_cast<const segment::CombineItem*>(tables + (plan.off_combine - plan.off_units));
  auto* corr_dev = reinterpret_cast<const segment::CorrItem*>(tables + (plan.off_corr - plan.off_units));
  CUtensorMap map_r{}, map_e{};
  if (!plan.corr.empty()) {  // R [tokens, hv, 128] and E [eslots * hv * 128 rows, 128] bf16, 128-row boxes
    uint64_t dims_r[3] = {kD, static_cast<uint64_t>(heads_v), static_cast<uint64_t>(total_tokens)};
    uint64_t strides_r[2] = {kD * 2, static_cast<uint64_t>(heads_v) * kD * 2};
    uint32_t box_r[3] = {64, 1, 128};
    uint64_t dims_e[2] = {kD, static_cast<uint64_t>(plan.num_eslots) * heads_v * kD};
    uint64_t strides_e[1] = {kD * 2};
    uint32_t box_e[2] = {64, 128};
    if (!encode_tiled(&map_r, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, r_out, dims_r, strides_r, box_r,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&map_e, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, e_bf16, dims_e, strides_e, box_e,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return TOKMIX_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (plan_dev == nullptr) {  // from host memory into the workspace (pageable: staged by the driver)
    std::vector<uint8_t> host(static_cast<size_t>(plan.total - plan.off_units));
    segment::write_tables(plan, host.data());
    if (cudaMemcpyAsync(ws + plan.off_units, host.data(), host.size(), cudaMemcpyHostToDevice, s) != cudaSuccess)
      return check_launch("tokmix_gdn_prefill_segmented: uploading the plan");
  }

  PrepParams pp{};
  pp.g = g;
  pp.beta = beta;
  pp.cu_seqlens = cu_seqlens_dev;
  pp.chunk_base = chunk_base_dev;
  pp.ws = ws;
  pp.num_seqs = num_seqs;
  pp.total_tokens = total_tokens;
  pp.hk = heads_k;
  pp.hv = heads_v;
  pp.scale = scale;
  pp.status = status;
  pp.gates = gate_source(gates);
  set_l2norm(pp, gates);
  if (total_chunks > 0) {
    const int smem = kPSmem + 1024;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&gdn_prep_kernel), smem))
      return check_launch("tokmix_gdn_prefill_segmented: cudaFuncSetAttribute (prep)");
    const int records = total_chunks * heads_v;
    const int grid = std::min(records, kPrepCtasPerSm * std::max(1, device_sm_count()));
    gdn_prep_kernel<<<grid, kPrepThreads, smem, s>>>(mq, mk, pp, records);
    if (const int rc = check_launch("tokmix_gdn_prefill_segmented (prep)")) return rc;
  }
  ChainParams cp{};
  cp.state_in = initial_state;
  cp.state_out = final_state;
  cp.checkpoints = nullptr;
  cp.out = static_cast<__nv_bfloat16*>(out);
  cp.cu_seqlens = cu_seqlens_dev;
  cp.chunk_base = chunk_base_dev;
  cp.ws = ws;
  cp.hk = heads_k;
  cp.hv = heads_v;
  cp.total_tokens = total_tokens;
  cp.total_chunks = total_chunks;
  cp.status = status;
  cp.units = units_dev;
  cp.num_units = static_cast<int>(plan.units.size());
  cp.num_slots = plan.num_slots;
  cp.num_seqs = num_seqs;
  cp.seg_states = seg_states;
  cp.r_out = r_out;
  {
    const int smem = kCSmem + 1024;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&gdn_chain_kernel), smem))
      return check_launch("tokmix_gdn_prefill_segmented: cudaFuncSetAttribute (chain)");
    gdn_chain_kernel<<<static_cast<unsigned>(plan.units.size() * heads_v), kChainThreads, smem, s>>>(mkc, mv, cp);
    if (const int rc = check_launch("tokmix_gdn_prefill_segmented (chain)")) return rc;
  }
  if (!plan.combine.empty()) {
    const int smem = segment::kCombineSmem;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&segment::combine_kernel), smem))
      return check_launch("tokmix_gdn_prefill_segmented: cudaFuncSetAttribute (combine)");
    segment::combine_kernel<<<dim3(static_cast<unsigned>(plan.combine.size()), static_cast<unsigned>(heads_v),
                                   kD / segment::kCombineRows),
                              segment::kCombineThreads, smem, s>>>(combine_dev, static_cast<int>(plan.combine.size()),
                                                                  seg_states, e_bf16, final_state, heads_v,
                                                                  plan.num_slots, plan.num_eslots, num_seqs, status);
    if (const int rc = check_launch("tokmix_gdn_prefill_segmented (combine)")) return rc;
  }
  if (!plan.corr.empty()) {
    const int smem = segment::kCorrSmem + 1024;
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&segment::correction_kernel), smem))
      return check_launch("tokmix_gdn_prefill_segmented: cudaFuncSetAttribute (correction)");
    segment::correction_kernel<<<dim3(static_cast<unsigned>(plan.corr.size()), static_cast<unsigned>(heads_v)),
                                 segment::kCorrThreads, smem, s>>>(map_r, map_e, corr_dev,
                                                                   static_cast<int>(plan.corr.size()),
                                                                   static_cast<__nv_bfloat16*>(out), heads_v,
                                                                   total_tokens, plan.num_eslots, status);
    if (const int rc = check_launch("tokmix_gdn_prefill_segmented (correction)")) return rc;
  }
  return TOKMIX_OK;
}
