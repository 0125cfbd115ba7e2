// gdn_segment.cuh -- the two stages that join the segments of a sequence after the record-fed
// chains have run them side by side (the segmented GDN schedule, host entry in gdn_split.cu).
//
// A sequence cut into segments 0..s-1 (at chunk boundaries) was chained as:
//   segment 0      from the sequence's initial state, outputs final, end state E_1
//   segment j >= 1 twice: from a zero state with the real V (outputs O_j^loc, end state N_j), and
//                  from the identity with V = 0 (outputs R_j, end state M_j).
// Because the state after any token is affine in the segment's entry state E_j (rows of the
// state evolve independently, S_t = E_j A_t + S_t^loc with A_t the product of the per-token
// transitions), the true quantities are
//   O_j = O_j^loc + R_j E_j^T          (per token t: o_t[v] += sum_i R_j[t][i] E_j[v][i])
//   E_{j+1} = E_j M_j + N_j            (E_s is the final state)
// combine_kernel walks j = 1..s-1 in fp32 (rows of E are independent, so a CTA owns 32 of them)
// and leaves E_j as bf16 for correction_kernel, a tcgen05 GEMM per 128-token tile that adds
// R_j E_j^T to the bf16 outputs in place.
#pragma once

#include <cuda_bf16.h>

#include "gdn_common.cuh"

namespace tokmix {
namespace gdn {
namespace segment {

// One segmented sequence: its state slots are slot_base + 0 (E_1), slot_base + 2j - 1 (N_j),
// slot_base + 2j (M_j) for j = 1..nseg-1; its bf16 entry states e_base + j - 1 (E_j).
struct CombineItem {
  int32_t seq, nseg, slot_base, e_base;
};

// One 128-token tile of a later segment: tokens [tok0, tok0 + ntok) use entry state e_slot.
struct CorrItem {
  int32_t tok0, ntok, e_slot, pad;
};

constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 32;  // rows of E per CTA
constexpr int kCombineSmem = kD * kD * 4 + kCombineRows * kD * 4;

// grid (items, hv, 128 / kCombineRows).  A CTA owns rows [v0, v0 + 32) of E; thread t computes
// the 4 x 8 tile rows v0 + 4 (t / 16) .. +3, columns 8 (t % 16) .. +7 of E_j M_j + N_j, reading
// per k one float4 of E (kept transposed in shared memory) and two of M_j.
__global__ void __launch_bounds__(kCombineThreads, 1)
    combine_kernel(const CombineItem* items, int num_items, const float* seg_states, __nv_bfloat16* e_bf16,
                   float* final_state, int hv, int num_slots, int num_eslots, int num_seqs, uint32_t* status) {
  extern __shared__ float4 smem_f4[];
  float* Ms = reinterpret_cast<float*>(smem_f4);   // M_j [k][c], 128 x 128
  float* Et = Ms + kD * kD;                         // E_j^T [k][r] for the block's 32 rows
  const int it = blockIdx.x, h = blockIdx.y, v0 = blockIdx.z * kCombineRows;
  const int t = threadIdx.x, r0 = (t >> 4) * 4, c0 = (t & 15) * 8;
  if (it >= num_items) return;
  const CombineItem ci = items[it];
  // device-resident table: reject what would index outside the buffers
  if (ci.seq < 0 || ci.seq >= num_seqs || ci.nseg < 2 || ci.slot_base < 0 || ci.slot_base + 2 * (ci.nseg - 1) >= num_slots ||
      ci.e_base < 0 || ci.e_base + ci.nseg - 1 > num_eslots) {
    if (t == 0) record_status(status, kDevBadArgs);
    return;
  }
  auto slot_ptr = [&](int slot) { return seg_states + (static_cast<size_t>(slot) * hv + h) * kD * kD; };
  float acc[4][8];  // rows r0..r0+3, columns c0..c0+7
  {  // E_1: the first segment's end state
    const float* e1 = slot_ptr(ci.slot_base) + (v0 + r0) * kD + c0;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(e1 + a * kD));
      const float4 y = __ldg(reinterpret_cast<const float4*>(e1 + a * kD + 4));
      acc[a][0] = x.x; acc[a][1] = x.y; acc[a][2] = x.z; acc[a][3] = x.w;
      acc[a][4] = y.x; acc[a][5] = y.y; acc[a][6] = y.z; acc[a][7] = y.w;
    }
  }
  for (int j = 1; j < ci.nseg; ++j) {
    __syncthreads();  // the previous step's reads of Et and Ms are done
    // E_j: transposed into shared memory, and as bf16 for the correction
#pragma unroll
    for (int a = 0; a < 4; ++a) {
#pragma unroll
      for (int e = 0; e < 8; ++e) Et[(c0 + e) * kCombineRows + r0 + a] = acc[a][e];
      __nv_bfloat16* dst = e_bf16 + (static_cast<size_t>(ci.e_base + j - 1) * hv + h) * kD * kD + (v0 + r0 + a) * kD + c0;
      *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(acc[a][0], acc[a][1]), pack_bf16x2(acc[a][2], acc[a][3]),
                                                  pack_bf16x2(acc[a][4], acc[a][5]), pack_bf16x2(acc[a][6], acc[a][7]));
    }
    // M_j to shared memory: 32 float4 per thread, 8 loads in flight at a time
    const float4* M4 = reinterpret_cast<const float4*>(slot_ptr(ci.slot_base + 2 * j));
    float4* Ms4 = reinterpret_cast<float4*>(Ms);
#pragma unroll 1
    for (int i0 = 0; i0 < kD * kD / 4; i0 += 8 * kCombineThreads) {
      float4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) buf[u] = __ldg(M4 + i0 + u * kCombineThreads + t);
#pragma unroll
      for (int u = 0; u < 8; ++u) Ms4[i0 + u * kCombineThreads + t] = buf[u];
    }
    // acc = N_j (the thread's tile), then += E_j M_j
    const float* Nr = slot_ptr(ci.slot_base + 2 * j - 1) + (v0 + r0) * kD + c0;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(Nr + a * kD));
      const float4 y = __ldg(reinterpret_cast<const float4*>(Nr + a * kD + 4));
      acc[a][0] = x.x; acc[a][1] = x.y; acc[a][2] = x.z; acc[a][3] = x.w;
      acc[a][4] = y.x; acc[a][5] = y.y; acc[a][6] = y.z; acc[a][7] = y.w;
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < kD; ++k) {
      const float4 ev = *reinterpret_cast<const float4*>(Et + k * kCombineRows + r0);
      const float4 m0 = *reinterpret_cast<const float4*>(Ms + k * kD + c0);
      const float4 m1 = *reinterpret_cast<const float4*>(Ms + k * kD + c0 + 4);
      const float e4[4] = {ev.x, ev.y, ev.z, ev.w};
      const float m8[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[a][e] = fmaf(e4[a], m8[e], acc[a][e]);
    }
  }
  float* fs = final_state + (static_cast<size_t>(ci.seq) * hv + h) * kD * kD + (v0 + r0) * kD + c0;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    *reinterpret_cast<float4*>(fs + a * kD) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    *reinterpret_cast<float4*>(fs + a * kD + 4) = make_float4(acc[a][4], acc[a][5], acc[a][6], acc[a][7]);
  }
}

constexpr int kCorrThreads = 128;
constexpr int kCorrSmem = 4 * 16384;  // R tile (two 64-column boxes of 128 rows) + E tile (same)

// grid (items, hv).  D[t][v] = sum_i R[tok0 + t][h][i] E[v][i] on the tensor core (M = 128
// tokens, N = 128 value rows, K = 128; both operands K-major, 128-byte swizzled boxes), then
// thread t adds row t of D to out[tok0 + t][h][:] (bf16) for t < ntok.
__global__ void __launch_bounds__(kCorrThreads, 1)
    correction_kernel(const __grid_constant__ CUtensorMap map_r, const __grid_constant__ CUtensorMap map_e,
                      const CorrItem* items, int num_items, __nv_bfloat16* out, int hv, int total_tokens, int num_eslots,
                      uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in, bar_mma, bar_drain;
  __shared__ uint32_t tmem_base_shared;
  const int it = blockIdx.x, h = blockIdx.y, t = threadIdx.x, warp = t >> 5;
  if (it >= num_items) return;
  const CorrItem ci = items[it];
  const bool bad = ci.tok0 < 0 || ci.ntok < 1 || ci.ntok > 128 || ci.tok0 > total_tokens - ci.ntok || ci.e_slot < 0 ||
                   ci.e_slot >= num_eslots;
  if (bad) {
    if (t == 0) record_status(status, kDevBadArgs);
    return;
  }
  if (t == 0) {
    cta_abort_flag() = 0u;
    mbar_init(&bar_in, 1);
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_shared, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_shared;
  const int erow = (ci.e_slot * hv + h) * kD;  // first row of E_j for head h in the 2-D map
  if (t == 0) {
    tma_prefetch_desc(&map_r);
    tma_prefetch_desc(&map_e);
    mbar_arrive_expect_tx(&bar_in, kCorrSmem);
    for (int bx = 0; bx < 2; ++bx) {
      tma_load_3d(smem + bx * 16384, &map_r, &bar_in, bx * 64, h, ci.tok0);
      tma_load_2d(smem + 32768 + bx * 16384, &map_e, &bar_in, bx * 64, erow);
    }
    bool ok = mbar_wait(&bar_in, 0, status, kDevTimeoutTma);
    if (ok) {
      tc_fence_after();
      const uint32_t id = make_idesc(128, 128, 1, 0, 0);
      const uint32_t a = smem_u32(smem), b = smem_u32(smem + 32768);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        umma_bf16_ss(tbase, make_sdesc_sw128(a + off, 16, 1024), make_sdesc_sw128(b + off, 16, 1024), id,
                     kk > 0 ? 1u : 0u);
      }
      umma_commit(&bar_mma);
    } else {
      mbar_drain(&bar_in, 0);  // let the copies land before the CTA retires
    }
  }
  __syncwarp();
  // the thread's output row is read while the operands load and the product runs
  uint4* orow = reinterpret_cast<uint4*>(out + (static_cast<size_t>(ci.tok0 + t) * hv + h) * kD);
  uint4 o[16];
  if (t < ci.ntok) {
#pragma unroll
    for (int q = 0; q < 16; ++q) o[q] = orow[q];
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar_mma, 0, status, kDevTimeoutMma));
  if (ok) {
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 32 columns at a time
      uint32_t d[32];
      tmem_ld32(tmem_addr(tbase, warp * 32, 32 * c), d);
      if (t < ci.ntok) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t* w = reinterpret_cast<uint32_t*>(&o[4 * c + q]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[e]));
            w[e] = pack_bf16x2(f.x + __uint_as_float(d[8 * q + 2 * e]), f.y + __uint_as_float(d[8 * q + 2 * e + 1]));
          }
          orow[4 * c + q] = o[4 * c + q];
        }
      }
    }
  }
  if (t == 0) {  // every MMA this thread issued completes before TMEM is released (bounded)
    umma_commit(&bar_drain);
    mbar_drain(&bar_drain, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

}  // namespace segment
}  // namespace gdn
}  // namespace tokmix
