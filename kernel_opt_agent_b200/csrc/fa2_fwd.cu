// fa2_fwd.cu -- causal / non-causal attention forward for sm_100a (B200).
//
// Reference path replaced: kernels_optimized/flash_attention_2.cu:814-1117 (the causal
// v4_tail kernel the reference dispatches to, :1243-1253) behind flash_attention_2_forward
// (:1121-1258).  Maths: references/flash_attention_2.py:27-41, i.e. torch SDPA with
// is_causal=causal and scale=sm_scale.
//
// Design (a work unit = one "pair" of 128-row query tiles that read the same keys/values; the
// launch is persistent, one CTA per SM walking its units heaviest first):
//   * pair = two query heads of one GQA group at the same query rows (heads_q/heads_kv even),
//     or two consecutive query tiles of one head (plain multi-head attention).  The K/V tiles
//     are loaded once per pair and used by both tiles' MMAs.
//   * warp 8 (one lane) issues TMA loads: the two Q tiles once, then K_j / V_j into a 2-stage
//     ring each (128 keys x head_dim bf16, 128B-swizzled boxes of 64 columns).
//   * warp 9 (one lane) owns TMEM (512 columns) and issues every tcgen05.mma:
//       S_i = Q_i K_j^T        (SS: both operands K-major in shared memory)      -> TMEM
//       O_i += P_i V_j         (TS: P_i read from TMEM, V_j MN-major in smem)    -> TMEM
//     in the order S_0(j) S_1(j) | PV_0(j) S_0(j+1) PV_1(j) S_1(j+1) | ... so the tensor core
//     works on one tile while the other tile's softmax runs.
//   * warps 0-3 / 4-7: softmax for tile 0 / 1.  Thread r owns query row r (TMEM lane r): it
//     reads its 128 scores, applies the causal / length mask, keeps a running max m and sum l
//     (base-2 domain), rescales O in TMEM only when the max grows by more than 2^8, writes
//     P = 2^(s*scale*log2e - m) as bf16 over the first 64 columns of its S region, and at the
//     end divides O by l and stores the bf16 row.
// TMEM columns: S_0 [0,128)  O_0 [128,128+D)  S_1 [256,384)  O_1 [384,384+D).
// Every wait is bounded (sm100.cuh): a stuck pipeline sets a status bit and the CTA drains.
// head_dim 256 has its own kernel (namespace d256 below): one query tile per unit, S double-buffered.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

#include "host_common.h"
#include "sm100.cuh"

namespace tokmix {
namespace fa2 {

constexpr int kBM = 128;        // query rows per tile
constexpr int kBN = 128;        // keys per kv tile
constexpr int kThreads = 320;   // 8 softmax warps + TMA warp + MMA warp
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

template <int D>
struct Layout {
  static constexpr int kTileBytes = kBM * D * 2;  // a Q, K or V tile: 128 rows x D bf16
  static constexpr int kBoxBytes = 128 * 128;     // one SW128 box: 128 rows x 64 bf16
  static constexpr int kQ0 = 0;
  static constexpr int kQ1 = kTileBytes;
  static constexpr int kK = 2 * kTileBytes;        // 2 stages
  static constexpr int kV = 4 * kTileBytes;        // 2 stages
  static constexpr int kBytes = 6 * kTileBytes;
  static constexpr int kColS0 = 0, kColO0 = 128, kColS1 = 256, kColO1 = 384;
};

struct Params {
  __nv_bfloat16* o;
  long long o_sb, o_sh, o_ss;  // element strides of the output (batch, head, seq)
  int batch, hq, hkv, sq, skv;
  int causal;
  float scale_log2;            // sm_scale * log2(e)
  int pair_heads;              // 1: a pair is two heads of one GQA group; 0: two query tiles of one head
  int n_qtiles;                // ceil(sq / 128)
  int head_units;              // pairs of heads (pair_heads) or heads
  int units;                   // work units (tile pairs), heaviest first
  uint32_t* status;
};

struct TileInfo {
  int head;     // query head
  int q0;       // first query row
  int n_kv;     // number of kv tiles this tile visits (0 = inactive)
};

// The r-th unit of this CTA in a persistent launch: units are heaviest first, and rounds of
// gridDim.x units go to the CTAs in alternating directions, so that every CTA's total stays
// within one unit of the others'.
__device__ __forceinline__ int unit_of_round(int r) {
  const int pos = (r & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  return r * static_cast<int>(gridDim.x) + pos;
}

__device__ __forceinline__ void decode_unit(const Params& p, int u, int& b, int& kvh, TileInfo (&t)[2]) {
  const int per_row = p.batch * p.head_units;
  const int rev = u / per_row;
  const int rem = u - rev * per_row;
  b = rem / p.head_units;
  const int hu = rem - b * p.head_units;
  const int group = p.hq / p.hkv;
  const int kv_tiles_all = (p.skv + kBN - 1) / kBN;
  if (p.pair_heads) {
    const int qt = p.n_qtiles - 1 - rev;
    for (int i = 0; i < 2; ++i) {
      t[i].head = 2 * hu + i;
      t[i].q0 = qt * kBM;
    }
  } else {
    const int npairs = (p.n_qtiles + 1) / 2;
    const int qp = npairs - 1 - rev;
    for (int i = 0; i < 2; ++i) {
      t[i].head = hu;
      t[i].q0 = (2 * qp + i) * kBM;
    }
  }
  kvh = t[0].head / group;
  for (int i = 0; i < 2; ++i) {
    if (t[i].q0 >= p.sq) {
      t[i].n_kv = 0;
    } else if (p.causal) {
      t[i].n_kv = min(kv_tiles_all, t[i].q0 / kBN + 1);
    } else {
      t[i].n_kv = kv_tiles_all;
    }
  }
}

// Persistent: CTA c takes its work units (tile pairs) round by round (unit_of_round), so barriers
// and TMEM are set up once per CTA and the next unit's Q load
// and first S MMAs run while the softmax warps finish the previous unit's epilogue.  Barrier
// phases carry over from unit to unit: the K/V ring by a running key-tile count g, bar_s/bar_p
// by each tile slot's running step count, bar_q, bar_qfree, bar_o and bar_ofree by unit.
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa2_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v, const Params p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_q, bar_qfree, bar_kfull[2], bar_kempty[2], bar_vfull[2], bar_vempty[2], bar_s[2], bar_p[2],
      bar_o[2], bar_ofree[2];
  __shared__ uint64_t bar_drain;
  __shared__ uint32_t tmem_base_shared;

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    mbar_init(&bar_q, 1);
    mbar_init(&bar_qfree, 1);
    mbar_init(&bar_drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_kfull[i], 1);
      mbar_init(&bar_kempty[i], 1);
      mbar_init(&bar_vfull[i], 1);
      mbar_init(&bar_vempty[i], 1);
      mbar_init(&bar_s[i], 1);
      mbar_init(&bar_p[i], 128);
      mbar_init(&bar_o[i], 1);
      mbar_init(&bar_ofree[i], 128);
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

  if (warp == kWarpTma) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      bool ok = true;
      int g = 0, it = 0;                          // key tiles and units begun
      int q_issued = 0, k_issued = 0, v_issued = 0;  // loads issued, for the drain
      for (int r = 0; ok; ++r, ++it) {
        const int u = unit_of_round(r);
        if (u >= p.units) break;
        int b, kvh;
        TileInfo tile[2];
        decode_unit(p, u, b, kvh, tile);
        const int nmax = max(tile[0].n_kv, tile[1].n_kv);
        // Q of this unit once the previous unit's last S MMAs have read the Q tiles
        if (it > 0 && !mbar_wait(&bar_qfree, (it - 1) & 1, p.status, kDevTimeoutPipe)) break;
        uint32_t qbytes = 0;
        for (int i = 0; i < 2; ++i) qbytes += tile[i].n_kv > 0 ? L::kTileBytes : 0;
        mbar_arrive_expect_tx(&bar_q, qbytes);
        for (int i = 0; i < 2; ++i) {
          if (tile[i].n_kv == 0) continue;
          uint8_t* dst = smem + (i == 0 ? L::kQ0 : L::kQ1);
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(dst + bx * L::kBoxBytes, &map_q, &bar_q, bx * 64, tile[i].q0, tile[i].head, b);
        }
        q_issued = it + 1;
        for (int j = 0; j < nmax; ++j, ++g) {
          const int st = g & 1;
          if (g >= 2 && !mbar_wait(&bar_kempty[st], ((g >> 1) - 1) & 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar_kfull[st], L::kTileBytes);
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(smem + L::kK + st * L::kTileBytes + bx * L::kBoxBytes, &map_k, &bar_kfull[st], bx * 64,
                        j * kBN, kvh, b);
          k_issued = g + 1;
          if (g >= 2 && !mbar_wait(&bar_vempty[st], ((g >> 1) - 1) & 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar_vfull[st], L::kTileBytes);
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(smem + L::kV + st * L::kTileBytes + bx * L::kBoxBytes, &map_v, &bar_vfull[st], bx * 64,
                        j * kBN, kvh, b);
          v_issued = g + 1;
        }
      }
      // before the CTA retires, let the last loads land (bounded; a no-op on the normal path)
      if (q_issued > 0) mbar_drain(&bar_q, (q_issued - 1) & 1);
      for (int t = max(0, k_issued - 2); t < k_issued; ++t) mbar_drain(&bar_kfull[t & 1], (t >> 1) & 1);
      for (int t = max(0, v_issued - 2); t < v_issued; ++t) mbar_drain(&bar_vfull[t & 1], (t >> 1) & 1);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc(kBM, kBN, 1, 0, 0);
      const uint32_t idesc_o = make_idesc(kBM, D, 1, 0, 1);
      const uint32_t col_s[2] = {static_cast<uint32_t>(L::kColS0), static_cast<uint32_t>(L::kColS1)};
      const uint32_t col_o[2] = {static_cast<uint32_t>(L::kColO0), static_cast<uint32_t>(L::kColO1)};
      const uint32_t q_addr[2] = {smem_u32(smem + L::kQ0), smem_u32(smem + L::kQ1)};
      auto issue_s = [&](int i, int st) {
        const uint32_t ka = smem_u32(smem + L::kK + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
          umma_bf16_ss(tbase + col_s[i], make_sdesc_sw128(q_addr[i] + off, 16, 1024),
                       make_sdesc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int i, int st, bool accumulate) {
        const uint32_t va = smem_u32(smem + L::kV + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_bf16_ts(tbase + col_o[i], tbase + col_s[i] + 8 * kk,
                       make_sdesc_sw128(va + kk * 2048, L::kBoxBytes, 1024), idesc_o,
                       (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      int g = 0, it = 0;         // key tiles of earlier units; units begun
      int steps[2] = {0, 0};     // each tile slot's steps in earlier units (bar_s, bar_p phases)
      int outs[2] = {0, 0};      // earlier units in which the slot was active (bar_o, bar_ofree phases)
      for (int r = 0; ok; ++r, ++it) {
        const int u = unit_of_round(r);
        if (u >= p.units) break;
        int b, kvh;
        TileInfo tile[2];
        decode_unit(p, u, b, kvh, tile);
        const int nmax = max(tile[0].n_kv, tile[1].n_kv);
        ok = mbar_wait(&bar_q, it & 1, p.status, kDevTimeoutTma) &&
             mbar_wait(&bar_kfull[g & 1], (g >> 1) & 1, p.status, kDevTimeoutTma);
        if (!ok) break;
        tc_fence_after();
        // S(0): S_i's columns were last read by the previous unit's PV_i, issued earlier by this thread
        for (int i = 0; i < 2; ++i) {
          if (tile[i].n_kv > 0) {
            issue_s(i, g & 1);
            umma_commit(&bar_s[i]);
          }
        }
        umma_commit(&bar_kempty[g & 1]);
        if (nmax == 1) umma_commit(&bar_qfree);  // no later S of this unit reads Q
        for (int j = 0; ok && j < nmax; ++j) {
          const int gj = g + j, st = gj & 1, gn = gj + 1, stn = gn & 1;
          if (!mbar_wait(&bar_vfull[st], (gj >> 1) & 1, p.status, kDevTimeoutTma)) { ok = false; break; }
          tc_fence_after();
          bool k_ready = false;
          for (int i = 0; i < 2 && ok; ++i) {
            if (j >= tile[i].n_kv) continue;
            if (!mbar_wait(&bar_p[i], (steps[i] + j) & 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
            // PV(0) overwrites O: the softmax warps have read the previous unit's O out of it
            if (j == 0 && outs[i] > 0 && !mbar_wait(&bar_ofree[i], (outs[i] - 1) & 1, p.status, kDevTimeoutPipe)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(i, st, j > 0);
            if (j == tile[i].n_kv - 1) umma_commit(&bar_o[i]);
            if (j + 1 < tile[i].n_kv) {
              if (!k_ready) {
                if (!mbar_wait(&bar_kfull[stn], (gn >> 1) & 1, p.status, kDevTimeoutTma)) { ok = false; break; }
                tc_fence_after();
                k_ready = true;
              }
              issue_s(i, stn);
              umma_commit(&bar_s[i]);
            }
          }
          if (!ok) break;
          umma_commit(&bar_vempty[st]);
          if (k_ready) umma_commit(&bar_kempty[stn]);
          if (j == nmax - 2) umma_commit(&bar_qfree);  // the unit's last S MMAs are issued
        }
        for (int i = 0; i < 2; ++i) {
          if (tile[i].n_kv > 0) {
            steps[i] += tile[i].n_kv;
            ++outs[i];
          }
        }
        g += nmax;
      }
      // every MMA issued by this thread completes before TMEM is released (bounded)
      umma_commit(&bar_drain);
      mbar_drain(&bar_drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int i = warp >> 2;
    const int qrow_local = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem_addr(tbase, (warp & 3) * 32, 0);
    const uint32_t col_s = i == 0 ? L::kColS0 : L::kColS1;
    const uint32_t col_o = i == 0 ? L::kColO0 : L::kColO1;
    const float c = p.scale_log2;
    bool ok = true;
    int steps = 0, outs = 0;  // this slot's steps and active units so far (barrier phases)
    for (int r = 0; ok; ++r) {
      const int u = unit_of_round(r);
      if (u >= p.units) break;
      int b, kvh;
      TileInfo tile[2];
      decode_unit(p, u, b, kvh, tile);
      const int n_kv = tile[i].n_kv;
      if (n_kv == 0) continue;  // the slot has no tile in this unit
      const int qrow = tile[i].q0 + qrow_local;
      float m = -INFINITY;
      float l = 0.0f;
      for (int j = 0; j < n_kv; ++j) {
        // tcgen05.ld/st are warp-collective: the whole warp continues or stops together
        if (!__all_sync(0xffffffffu, mbar_wait(&bar_s[i], (steps + j) & 1, p.status, kDevTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t raw[128];
        tmem_ld64(lane_base + col_s, *reinterpret_cast<uint32_t(*)[64]>(&raw[0]));
        tmem_ld64(lane_base + col_s + 64, *reinterpret_cast<uint32_t(*)[64]>(&raw[64]));
        float s[128];
  #pragma unroll
        for (int cc = 0; cc < 128; ++cc) s[cc] = __uint_as_float(raw[cc]);
        const int kv0 = j * kBN;
        const bool need_mask = (p.causal && kv0 + kBN - 1 > tile[i].q0) || (kv0 + kBN > p.skv);
        if (need_mask) {
          const int lim = (p.causal ? min(qrow + 1, p.skv) : p.skv) - kv0;
  #pragma unroll
          for (int cc = 0; cc < 128; ++cc)
            if (cc >= lim) s[cc] = -INFINITY;
        }
        float mx;
        {  // four independent chains of three-input maxima over the 128 columns
          float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
  #pragma unroll
          for (int cc = 0; cc < 128; cc += 8) {
            m0 = max3f(m0, s[cc], s[cc + 1]);
            m1 = max3f(m1, s[cc + 2], s[cc + 3]);
            m2 = max3f(m2, s[cc + 4], s[cc + 5]);
            m3 = max3f(m3, s[cc + 6], s[cc + 7]);
          }
          mx = max3f(m0, m1, fmaxf(m2, m3));
        }
        const float mx_scaled = mx * c;
        // Lazy rescale: a row moves its running max only when it grew by more than 2^8.  The
        // decision is per row, the O read-modify-write is done by the whole warp (alpha = 1 for
        // rows that keep their max) because tcgen05.ld/st are warp-collective.
        const bool grow = mx_scaled > m + kRescaleThreshold;
        float alpha = 1.0f;
        if (grow) {
          alpha = ex2_approx(m - mx_scaled);
          m = mx_scaled;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O holds sum_{<j} P V; PV(j-1) is complete because S(j) was committed after it.
  #pragma unroll 1
          for (int dc = 0; dc < D; dc += 32) {
            uint32_t o_raw[32];
            tmem_ld32(lane_base + col_o + dc, o_raw);
  #pragma unroll
            for (int e = 0; e < 32; ++e) o_raw[e] = __float_as_uint(__uint_as_float(o_raw[e]) * alpha);
            tmem_st32(lane_base + col_o + dc, o_raw);
          }
        }
        l *= alpha;
        float rowsum = 0.0f;
  #pragma unroll
        for (int chunk = 0; chunk < 4; ++chunk) {
          uint32_t packed[16];
  #pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = ex2_approx(fmaf(s[chunk * 32 + 2 * e], c, -m));
            const float p1 = ex2_approx(fmaf(s[chunk * 32 + 2 * e + 1], c, -m));
            rowsum += p0 + p1;
            packed[e] = pack_bf16x2(p0, p1);
          }
          tmem_st16(lane_base + col_s + chunk * 16, packed);
        }
        l += rowsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bar_p[i]);
      }
      if (!ok) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_o[i], outs & 1, p.status, kDevTimeoutMma))) {
        ok = false;
        break;
      }
      {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* orow = p.o + static_cast<long long>(b) * p.o_sb + static_cast<long long>(tile[i].head) * p.o_sh +
                              static_cast<long long>(qrow) * p.o_ss;
  #pragma unroll 1
        for (int dc = 0; dc < D; dc += 32) {
          uint32_t o_raw[32];
          tmem_ld32(lane_base + col_o + dc, o_raw);
          uint32_t packed[16];
  #pragma unroll
          for (int e = 0; e < 16; ++e)
            packed[e] = pack_bf16x2(__uint_as_float(o_raw[2 * e]) * inv_l, __uint_as_float(o_raw[2 * e + 1]) * inv_l);
          if (qrow < p.sq) {
            uint4* dst = reinterpret_cast<uint4*>(orow + dc);
  #pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(packed[4 * v4], packed[4 * v4 + 1], packed[4 * v4 + 2], packed[4 * v4 + 3]);
          }
        }
      }
      // the O columns are read (tcgen05.ld waited): the next unit's PV may overwrite them
      tc_fence_before();
      mbar_arrive(&bar_ofree[i]);
      steps += n_kv;
      ++outs;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

template <int D>
int launch(const void* q, const void* k, const void* v, void* o, int batch, int hq, int hkv, int sq, int skv,
           int layout, int causal, float sm_scale, uint32_t* status, cudaStream_t stream) {
  using L = Layout<D>;
  // 4-D tensor maps over (d, seq, head, batch); the layout only changes the strides.
  auto make = [&](CUtensorMap* map, const void* base, int s, int h) {
    uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(s), static_cast<uint64_t>(h),
                        static_cast<uint64_t>(batch)};
    uint64_t strides[3];
    const uint64_t row = static_cast<uint64_t>(D) * 2;
    if (layout == TOKMIX_LAYOUT_BHSD) {
      strides[0] = row;
      strides[1] = row * s;
      strides[2] = row * s * h;
    } else {
      strides[0] = row * h;
      strides[1] = row;
      strides[2] = row * s * h;
    }
    uint32_t box[4] = {64, 128, 1, 1};
    return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap mq, mk, mv;
  if (!make(&mq, q, sq, hq) || !make(&mk, k, skv, hkv) || !make(&mv, v, skv, hkv)) return TOKMIX_ERR_INVALID_ARGUMENT;

  Params p{};
  p.o = static_cast<__nv_bfloat16*>(o);
  if (layout == TOKMIX_LAYOUT_BHSD) {
    p.o_ss = D;
    p.o_sh = static_cast<long long>(D) * sq;
    p.o_sb = static_cast<long long>(D) * sq * hq;
  } else {
    p.o_sh = D;
    p.o_ss = static_cast<long long>(D) * hq;
    p.o_sb = static_cast<long long>(D) * sq * hq;
  }
  p.batch = batch;
  p.hq = hq;
  p.hkv = hkv;
  p.sq = sq;
  p.skv = skv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  const int group = hq / hkv;
  p.pair_heads = (group % 2 == 0) ? 1 : 0;
  p.n_qtiles = (sq + kBM - 1) / kBM;
  p.head_units = p.pair_heads ? hq / 2 : hq;
  p.status = status;
  const long long rows = p.pair_heads ? p.n_qtiles : (p.n_qtiles + 1) / 2;
  const long long units = rows * batch * p.head_units;
  if (units <= 0) return TOKMIX_OK;
  if (units > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_fa2_fwd: too many tiles (%lld)", units);

  p.units = static_cast<int>(units);
  const int smem_bytes = L::kBytes + 1024;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(&fa2_fwd_kernel<D>), smem_bytes))
    return check_launch("tokmix_fa2_fwd: cudaFuncSetAttribute");
  const int grid = static_cast<int>(std::min<long long>(units, std::max(1, device_sm_count())));
  fa2_fwd_kernel<D><<<static_cast<unsigned>(grid), kThreads, smem_bytes, stream>>>(mq, mk, mv, p);
  return check_launch("tokmix_fa2_fwd");
}

// ---------------------------------------------------------------------------------------------
// head_dim 256.  Two tiles' S and O (2 x (128 + 256) TMEM columns) do not fit in TMEM, so a work
// unit is one 128-row query tile, and S is double-buffered instead: the tensor core computes S(j+1)
// while the softmax warps work on S(j).  Keys come in tiles of 128 (S(j) is one N=128 product
// per 16-column step of Q, PV(j) a K=128 product), with K(j) and V(j) single-buffered (64 KB
// each; Q 64 KB: 192 KB of shared memory).  Order of the MMAs: S(0) | S(1) PV(0) | S(2) PV(1) |
// ...; S(j+1) overwrites the buffer PV(j-1) read P(j-1) from, after PV(j-1) in issue order.  The
// loads of K(j+1) start once S(j) has completed (while the softmax works on S(j)), those of V(j+1)
// once PV(j) has completed; one producer lane each, so neither waits behind the other's release.
// The lazy O rescale of step j needs PV(j-1) complete (it may still accumulate into O): the
// softmax warps then wait for its commit, which a rescale makes rare.
// Warps 0-3: softmax (thread = query row); warp 4: TMA (lane 0 Q and K, lane 1 V); warp 5: TMEM
// owner and MMA issuer.  TMEM columns: S0 [0,128)  S1 [128,256)  O [256,512).
// ---------------------------------------------------------------------------------------------
namespace d256 {

constexpr int kD = 256;
constexpr int kBN = 128;                           // keys per kv tile
constexpr int kThreads = 192;
constexpr int kWarpTma = 4, kWarpMma = 5;
constexpr int kQBytes = kBM * kD * 2;              // 64 KB: four boxes of 128 rows x 64 columns
constexpr int kQBox = kBM * 128;                   // 16 KB
constexpr int kKVBytes = kBN * kD * 2;             // 64 KB: four boxes of 128 rows x 64 columns
constexpr int kKVBox = kBN * 128;                  // 16 KB
constexpr int kQ = 0, kK = kQBytes, kV = kQBytes + kKVBytes, kBytes = kQBytes + 2 * kKVBytes;
static_assert(kBytes + 1024 <= 227 * 1024, "d256 shared memory budget");
__device__ __forceinline__ uint32_t col_s(int st) { return st ? 128u : 0u; }  // S buffer st
constexpr uint32_t kColO = 256;

// The unit u of the head_dim-256 launch: one 128-row query tile of one (batch, head), the heaviest
// (last) causal tiles first
__device__ __forceinline__ void decode_d256(const Params& p, int u, int& b, int& head, int& kvh, int& q0, int& n_kv) {
  const int per_row = p.batch * p.hq;
  const int rev = u / per_row;
  const int rem = u - rev * per_row;
  b = rem / p.hq;
  head = rem - b * p.hq;
  kvh = head / (p.hq / p.hkv);
  q0 = (p.n_qtiles - 1 - rev) * kBM;
  const int kv_tiles_all = (p.skv + kBN - 1) / kBN;
  n_kv = p.causal ? min(kv_tiles_all, (q0 + kBM - 1) / kBN + 1) : kv_tiles_all;
}

// Persistent like fa2_fwd_kernel: CTA c takes its units round by round (unit_of_round); the
// steps of all its units form one sequence g (S buffer g & 1, K and V tile g), so barrier phases
// carry over; the next unit's Q loads once the current unit's last S is issued (bar_qfree) and
// its first PV waits until the softmax warps have read the previous O out (bar_ofree).
__global__ void __launch_bounds__(kThreads, 1)
    fa2_fwd_d256_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_q, bar_qfree, bar_kfull, bar_kempty, bar_vfull, bar_vempty, bar_s[2], bar_p[2], bar_pv[2];
  __shared__ uint64_t bar_o, bar_ofree, bar_drain;
  __shared__ uint32_t tmem_base_shared;

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    mbar_init(&bar_q, 1);
    mbar_init(&bar_qfree, 1);
    mbar_init(&bar_o, 1);
    mbar_init(&bar_ofree, 128);
    mbar_init(&bar_drain, 1);
    mbar_init(&bar_kfull, 1);
    mbar_init(&bar_kempty, 1);
    mbar_init(&bar_vfull, 1);
    mbar_init(&bar_vempty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s[i], 1);
      mbar_init(&bar_p[i], 128);
      mbar_init(&bar_pv[i], 1);
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

  if (warp == kWarpTma) {
    // ------------------------------------------------------------------ TMA producers
    // K(g) waits for S(g-1) to release the K buffer, V(g) for PV(g-1) (kempty / vempty complete
    // once per tile, so the release of tile g-1 is phase (g-1) & 1)
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      bool ok = true;
      int g = 0, q_issued = 0, k_issued = 0;
      for (int r = 0; ok; ++r) {
        const int u = unit_of_round(r);
        if (u >= p.units) break;
        int b, head, kvh, q0, n_kv;
        decode_d256(p, u, b, head, kvh, q0, n_kv);
        if (r > 0 && !mbar_wait(&bar_qfree, (r - 1) & 1, p.status, kDevTimeoutPipe)) break;
        mbar_arrive_expect_tx(&bar_q, kQBytes);
        for (int bx = 0; bx < kD / 64; ++bx) tma_load_4d(smem + kQ + bx * kQBox, &map_q, &bar_q, bx * 64, q0, head, b);
        q_issued = r + 1;
        for (int j = 0; j < n_kv; ++j, ++g) {
          if (g >= 1 && !mbar_wait(&bar_kempty, (g - 1) & 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar_kfull, kKVBytes);
          for (int bx = 0; bx < kD / 64; ++bx)
            tma_load_4d(smem + kK + bx * kKVBox, &map_k, &bar_kfull, bx * 64, j * kBN, kvh, b);
          k_issued = g + 1;
        }
      }
      if (q_issued > 0) mbar_drain(&bar_q, (q_issued - 1) & 1);
      if (k_issued > 0) mbar_drain(&bar_kfull, (k_issued - 1) & 1);
    } else if (lane == 1) {
      tma_prefetch_desc(&map_v);
      bool ok = true;
      int g = 0, v_issued = 0;
      for (int r = 0; ok; ++r) {
        const int u = unit_of_round(r);
        if (u >= p.units) break;
        int b, head, kvh, q0, n_kv;
        decode_d256(p, u, b, head, kvh, q0, n_kv);
        for (int j = 0; j < n_kv; ++j, ++g) {
          if (g >= 1 && !mbar_wait(&bar_vempty, (g - 1) & 1, p.status, kDevTimeoutPipe)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar_vfull, kKVBytes);
          for (int bx = 0; bx < kD / 64; ++bx)
            tma_load_4d(smem + kV + bx * kKVBox, &map_v, &bar_vfull, bx * 64, j * kBN, kvh, b);
          v_issued = g + 1;
        }
      }
      if (v_issued > 0) mbar_drain(&bar_vfull, (v_issued - 1) & 1);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc(kBM, kBN, 1, 0, 0);
      const uint32_t idesc_o = make_idesc(kBM, kD, 1, 0, 1);
      const uint32_t qa = smem_u32(smem + kQ);
      const uint32_t ka = smem_u32(smem + kK);
      const uint32_t va = smem_u32(smem + kV);
      // S(g) = Q K(g)^T into S buffer g & 1, once K(g) is in; releases the K buffer
      auto issue_s = [&](int g) -> bool {
        if (!mbar_wait(&bar_kfull, g & 1, p.status, kDevTimeoutTma)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_bf16_ss(tbase + col_s(g & 1), make_sdesc_sw128(qa + (kk >> 2) * kQBox + (kk & 3) * 32, 16, 1024),
                       make_sdesc_sw128(ka + (kk >> 2) * kKVBox + (kk & 3) * 32, 16, 1024), idesc_s,
                       kk > 0 ? 1u : 0u);
        umma_commit(&bar_s[g & 1]);
        umma_commit(&bar_kempty);
        return true;
      };
      bool ok = true;
      int gbase = 0;  // steps of earlier units
      for (int r = 0; ok; ++r) {
        const int u = unit_of_round(r);
        if (u >= p.units) break;
        int b, head, kvh, q0, n_kv;
        decode_d256(p, u, b, head, kvh, q0, n_kv);
        ok = mbar_wait(&bar_q, r & 1, p.status, kDevTimeoutTma) && issue_s(gbase);
        if (ok && n_kv == 1) umma_commit(&bar_qfree);  // no later S of this unit reads Q
        for (int j = 0; ok && j < n_kv; ++j) {
          const int g = gbase + j, st = g & 1;
          // S(g+1) first: it runs while the softmax warps work on S(g)
          if (j + 1 < n_kv) {
            if (!issue_s(g + 1)) {
              ok = false;
              break;
            }
            if (j + 2 == n_kv) umma_commit(&bar_qfree);  // the unit's last S is issued
          }
          ok = mbar_wait(&bar_vfull, g & 1, p.status, kDevTimeoutTma) &&
               mbar_wait(&bar_p[st], (g >> 1) & 1, p.status, kDevTimeoutPipe);
          // PV(0) overwrites O: the softmax warps have read the previous unit's O out of it
          if (ok && j == 0 && r > 0) ok = mbar_wait(&bar_ofree, (r - 1) & 1, p.status, kDevTimeoutPipe);
          if (!ok) break;
          tc_fence_after();
          // O (+)= P(g) V(g): P read from TMEM (bf16 over S buffer g & 1), V MN-major in smem
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)
            umma_bf16_ts(tbase + kColO, tbase + col_s(st) + 8 * kk, make_sdesc_sw128(va + kk * 2048, kKVBox, 1024),
                         idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&bar_pv[st]);
          umma_commit(&bar_vempty);
          if (j == n_kv - 1) umma_commit(&bar_o);
        }
        gbase += n_kv;
      }
      umma_commit(&bar_drain);
      mbar_drain(&bar_drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax warps 0-3
    const int qrow_local = warp * 32 + lane;
    const uint32_t lane_base = tmem_addr(tbase, warp * 32, 0);
    const float c = p.scale_log2;
    bool ok = true;
    int gbase = 0;  // steps of earlier units
    for (int r = 0; ok; ++r) {
      const int u = unit_of_round(r);
      if (u >= p.units) break;
      int b, head, kvh, q0, n_kv;
      decode_d256(p, u, b, head, kvh, q0, n_kv);
      const int qrow = q0 + qrow_local;
      float m = -INFINITY;
      float l = 0.0f;
      for (int j = 0; j < n_kv; ++j) {
        const int g = gbase + j, st = g & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&bar_s[st], (g >> 1) & 1, p.status, kDevTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t raw[128];
        tmem_ld64(lane_base + col_s(st), *reinterpret_cast<uint32_t(*)[64]>(&raw[0]));
        tmem_ld64(lane_base + col_s(st) + 64, *reinterpret_cast<uint32_t(*)[64]>(&raw[64]));
        float s[128];
  #pragma unroll
        for (int cc = 0; cc < 128; ++cc) s[cc] = __uint_as_float(raw[cc]);
        const int kv0 = j * kBN;
        if ((p.causal && kv0 + kBN - 1 > q0) || (kv0 + kBN > p.skv)) {
          const int lim = (p.causal ? min(qrow + 1, p.skv) : p.skv) - kv0;
  #pragma unroll
          for (int cc = 0; cc < 128; ++cc)
            if (cc >= lim) s[cc] = -INFINITY;
        }
        float mx;
        {  // four independent chains of three-input maxima over the 128 columns
          float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
  #pragma unroll
          for (int cc = 0; cc < 128; cc += 8) {
            m0 = max3f(m0, s[cc], s[cc + 1]);
            m1 = max3f(m1, s[cc + 2], s[cc + 3]);
            m2 = max3f(m2, s[cc + 4], s[cc + 5]);
            m3 = max3f(m3, s[cc + 6], s[cc + 7]);
          }
          mx = max3f(m0, m1, fmaxf(m2, m3));
        }
        const float mx_scaled = mx * c;
        const bool grow = mx_scaled > m + kRescaleThreshold;
        float alpha = 1.0f;
        if (grow) {
          alpha = ex2_approx(m - mx_scaled);
          m = mx_scaled;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O holds sum_{<j} P V once PV(j-1) has completed
          if (!__all_sync(0xffffffffu, mbar_wait(&bar_pv[(g - 1) & 1], ((g - 1) >> 1) & 1, p.status, kDevTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
  #pragma unroll 1
          for (int dc = 0; dc < kD; dc += 32) {
            uint32_t o_raw[32];
            tmem_ld32(lane_base + kColO + dc, o_raw);
  #pragma unroll
            for (int e = 0; e < 32; ++e) o_raw[e] = __float_as_uint(__uint_as_float(o_raw[e]) * alpha);
            tmem_st32(lane_base + kColO + dc, o_raw);
          }
        }
        l *= alpha;
        float rowsum = 0.0f;
  #pragma unroll
        for (int chunk = 0; chunk < 4; ++chunk) {
          uint32_t packed[16];
  #pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = ex2_approx(fmaf(s[chunk * 32 + 2 * e], c, -m));
            const float p1 = ex2_approx(fmaf(s[chunk * 32 + 2 * e + 1], c, -m));
            rowsum += p0 + p1;
            packed[e] = pack_bf16x2(p0, p1);
          }
          tmem_st16(lane_base + col_s(st) + chunk * 16, packed);
        }
        l += rowsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bar_p[st]);
      }
      if (!ok) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_o, r & 1, p.status, kDevTimeoutMma))) {
        ok = false;
        break;
      }
      {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* orow = p.o + static_cast<long long>(b) * p.o_sb + static_cast<long long>(head) * p.o_sh +
                              static_cast<long long>(qrow) * p.o_ss;
  #pragma unroll 1
        for (int dc = 0; dc < kD; dc += 32) {
          uint32_t o_raw[32];
          tmem_ld32(lane_base + kColO + dc, o_raw);
          uint32_t packed[16];
  #pragma unroll
          for (int e = 0; e < 16; ++e)
            packed[e] = pack_bf16x2(__uint_as_float(o_raw[2 * e]) * inv_l, __uint_as_float(o_raw[2 * e + 1]) * inv_l);
          if (qrow < p.sq) {
            uint4* dst = reinterpret_cast<uint4*>(orow + dc);
  #pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(packed[4 * v4], packed[4 * v4 + 1], packed[4 * v4 + 2], packed[4 * v4 + 3]);
          }
        }
      }
      // the O columns are read (tcgen05.ld waited): the next unit's PV may overwrite them
      tc_fence_before();
      mbar_arrive(&bar_ofree);
      gbase += n_kv;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

int launch(const void* q, const void* k, const void* v, void* o, int batch, int hq, int hkv, int sq, int skv,
           int layout, int causal, float sm_scale, uint32_t* status, cudaStream_t stream) {
  auto make = [&](CUtensorMap* map, const void* base, int s, int h, uint32_t rows) {
    uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(s), static_cast<uint64_t>(h),
                        static_cast<uint64_t>(batch)};
    uint64_t strides[3];
    const uint64_t row = static_cast<uint64_t>(kD) * 2;
    if (layout == TOKMIX_LAYOUT_BHSD) {
      strides[0] = row;
      strides[1] = row * s;
      strides[2] = row * s * h;
    } else {
      strides[0] = row * h;
      strides[1] = row;
      strides[2] = row * s * h;
    }
    uint32_t box[4] = {64, rows, 1, 1};
    return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap mq, mk, mv;
  if (!make(&mq, q, sq, hq, kBM) || !make(&mk, k, skv, hkv, kBN) || !make(&mv, v, skv, hkv, kBN))
    return TOKMIX_ERR_INVALID_ARGUMENT;
  Params p{};
  p.o = static_cast<__nv_bfloat16*>(o);
  if (layout == TOKMIX_LAYOUT_BHSD) {
    p.o_ss = kD;
    p.o_sh = static_cast<long long>(kD) * sq;
    p.o_sb = static_cast<long long>(kD) * sq * hq;
  } else {
    p.o_sh = kD;
    p.o_ss = static_cast<long long>(kD) * hq;
    p.o_sb = static_cast<long long>(kD) * sq * hq;
  }
  p.batch = batch;
  p.hq = hq;
  p.hkv = hkv;
  p.sq = sq;
  p.skv = skv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.n_qtiles = (sq + kBM - 1) / kBM;
  p.status = status;
  const long long units = static_cast<long long>(p.n_qtiles) * batch * hq;
  if (units <= 0) return TOKMIX_OK;
  if (units > 0x7FFFFFFFll) return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_fa2_fwd: too many tiles (%lld)", units);
  const int smem_bytes = kBytes + 1024;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(&fa2_fwd_d256_kernel), smem_bytes))
    return check_launch("tokmix_fa2_fwd: cudaFuncSetAttribute");
  p.units = static_cast<int>(units);
  const int grid = static_cast<int>(std::min<long long>(units, std::max(1, device_sm_count())));
  fa2_fwd_d256_kernel<<<static_cast<unsigned>(grid), kThreads, smem_bytes, stream>>>(mq, mk, mv, p);
  return check_launch("tokmix_fa2_fwd (head_dim 256)");
}

}  // namespace d256

}  // namespace fa2
}  // namespace tokmix

extern "C" int tokmix_fa2_fwd(const void* q, const void* k, const void* v, void* o, int batch, int heads_q,
                              int heads_kv, int seqlen_q, int seqlen_kv, int head_dim, int layout, int causal,
                              float sm_scale, uint32_t* status, void* stream) {
  using namespace tokmix;
  if (batch < 0 || heads_q <= 0 || heads_kv <= 0 || seqlen_q < 0 || seqlen_kv < 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: negative or zero size");
  if (batch == 0 || seqlen_q == 0) return TOKMIX_OK;
  if (!q || !k || !v || !o) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: null tensor pointer");
  if (heads_q % heads_kv != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: heads_q (%d) must be a multiple of heads_kv (%d)",
                heads_q, heads_kv);
  if (layout != TOKMIX_LAYOUT_BHSD && layout != TOKMIX_LAYOUT_BSHD)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: unknown layout %d", layout);
  if (!(sm_scale > 0.0f) || !std::isfinite(sm_scale))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: sm_scale must be finite and positive");
  for (const void* ptr : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: tensors must be 16-byte aligned");
  if (const int rc = check_device()) return rc;
  if (seqlen_kv == 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_fa2_fwd: seqlen_kv must be positive when seqlen_q is");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64:
      return fa2::launch<64>(q, k, v, o, batch, heads_q, heads_kv, seqlen_q, seqlen_kv, layout, causal, sm_scale,
                             status, s);
    case 128:
      return fa2::launch<128>(q, k, v, o, batch, heads_q, heads_kv, seqlen_q, seqlen_kv, layout, causal, sm_scale,
                              status, s);
    case 256:
      return fa2::d256::launch(q, k, v, o, batch, heads_q, heads_kv, seqlen_q, seqlen_kv, layout, causal, sm_scale,
                               status, s);
    default:
      return fail(TOKMIX_ERR_UNSUPPORTED, "tokmix_fa2_fwd: head_dim %d not supported (64, 128 or 256)", head_dim);
  }
}
