// sm100.cuh -- thin inline-PTX layer over the Blackwell (sm_100a) features the token-mixer
// kernels are built on: mbarriers with bounded waits, TMA tiled loads, tcgen05 (TMEM alloc,
// UMMA issue/commit, TMEM <-> register moves) and the shared-memory / instruction descriptors
// the UMMA needs.  Everything here is written against the public PTX ISA; no CUDA math library
// code is restated.
//
// Conventions used by every kernel in this library:
//   * operand tiles live in shared memory in the 128-byte-swizzled canonical UMMA layout, the
//     same byte order a TMA load with CU_TENSOR_MAP_SWIZZLE_128B produces: a "row" is 128 bytes
//     (64 bf16 or 32 fp32), rows are packed back to back, and the 16-byte chunk c of row r sits
//     at chunk position c ^ (r % 8).  Tiles start on 1024-byte boundaries.
//   * waits never spin forever: every mbarrier wait gives up after kWaitTimeoutNs of wall time,
//     records a status code in the caller's device status word and returns false.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace tokmix {

// ------------------------------------------------------------------------------------------
// status codes written into the device status word (also returned by the C ABI)
// ------------------------------------------------------------------------------------------
enum DeviceStatus : uint32_t {
  kDevOk = 0,
  kDevTimeoutTma = 1u << 0,     // a TMA transaction barrier never completed
  kDevTimeoutMma = 1u << 1,     // a tcgen05 commit never arrived
  kDevTimeoutPipe = 1u << 2,    // a producer/consumer hand-off between warps never arrived
  kDevBadArgs = 1u << 3,        // a kernel-side argument check failed
};

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s of wall time

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(uint32_t* status, uint32_t code) {
  if (status != nullptr) atomicOr(status, code);
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival on behalf of `count` threads (used by one lane for its whole warp after __syncwarp)
__device__ __forceinline__ void mbar_arrive_count(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Potentially blocking test: the hardware may suspend the thread for a short while if the phase
// has not completed yet.  Used inside wait loops.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test, for a thread that polls several barriers and must not park on one of them.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Blocking test with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or `hint_ns` passes, so waiting warps take no issue slots or shared-memory bandwidth.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// CTA-wide abort flag in shared memory: set by the first wait that runs out, checked by every
// other wait so the whole CTA drains quickly.  Kernels zero it before their first barrier.
__device__ __forceinline__ volatile uint32_t& cta_abort_flag() {
  __shared__ uint32_t flag;
  return *reinterpret_cast<volatile uint32_t*>(&flag);
}

// Wait until the phase with the given parity has completed.  Gives up after `limit_ns` of wall
// time (kWaitTimeoutNs in every kernel; a shorter limit only in the wait self-test), records
// `code` in *status (device memory, may be null), raises the CTA abort flag and returns false;
// returns false at once if another warp of the CTA has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                          unsigned long long limit_ns = kWaitTimeoutNs) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_sleep(bar, parity, 100000u)) return true;
    if (cta_abort_flag() != 0u) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      record_status(status, code);
      cta_abort_flag() = 1u;
      return false;
    }
  }
}

// Bounded wait for a ready flag in global memory (written by another CTA of the same launch with
// release semantics); afterwards what the flag guards may be read through the async proxy.  Gives
// up like mbar_wait, recording kDevTimeoutPipe.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t* status,
                                          unsigned long long limit_ns = kWaitTimeoutNs) {
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v != 0u) break;
    if (cta_abort_flag() != 0u) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      record_status(status, kDevTimeoutPipe);
      cta_abort_flag() = 1u;
      return false;
    }
    __nanosleep(128);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Bounded wait that ignores the abort flag: used before a CTA retires, to let its own TMA loads
// and MMAs land before shared memory and TMEM are released.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_sleep(bar, parity, 100000u)) {
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return false;
  }
  return true;
}

// ------------------------------------------------------------------------------------------
// TMA (every load has one destination CTA)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Named barrier over `nthreads` threads that also ANDs a predicate across them: every thread
// gets the same answer, so a group can agree to stop together instead of leaving some threads
// parked at a barrier the others will never reach.
__device__ __forceinline__ bool named_sync_and(int id, int nthreads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}\n"
      : "=r"(out)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return out != 0;
}

// generic-proxy writes to shared memory -> visible to the async proxy (UMMA operand reads)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ------------------------------------------------------------------------------------------
// Whole warp must call.  Writes the TMEM base address into *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM address: lane in bits [31:16], column in bits [15:0]
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ------------------------------------------------------------------------------------------
// tcgen05: UMMA issue / commit (single thread)
// ------------------------------------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T   (kind::f16: bf16/fp16 operands, fp32 accumulate)
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::tf32: fp32 operands in shared memory (rounded to tf32 by the tensor core)
__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on *bar when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------------------------------
// descriptors
// ------------------------------------------------------------------------------------------
// Instruction descriptor for kind::f16 / kind::tf32 with fp32 accumulation.
//   ab_format: 0 = f16, 1 = bf16, 2 = tf32
//   a_mn_major / b_mn_major: 0 = K-major, 1 = MN-major
__host__ __device__ constexpr uint32_t make_idesc(uint32_t m, uint32_t n, uint32_t ab_format, uint32_t a_mn_major,
                                                  uint32_t b_mn_major, uint32_t negate_b = 0) {
  return (1u << 4)                   // D format: f32
         | (ab_format << 7)          // A format
         | (ab_format << 10)         // B format
         | (negate_b << 14)          // negate B
         | (a_mn_major << 15)        // A major
         | (b_mn_major << 16)        // B major
         | ((n >> 3) << 17)          // N / 8
         | ((m >> 4) << 24);         // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle.
//   K-major operand:  sbo = byte distance between consecutive 8-row groups (1024 for packed rows);
//                     lbo is ignored by the hardware (encoded as 16 bytes).
//   MN-major operand: lbo = byte distance between consecutive 64-element (128 B) chunks along MN,
//                     sbo = byte distance between consecutive 8-row groups along K.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Byte offset of element (row, byte_in_row) inside a 128B-swizzled tile whose rows are 128 bytes.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t byte_in_row) {
  return row * 128u + ((((byte_in_row >> 4) ^ (row & 7u)) << 4) | (byte_in_row & 15u));
}

// ------------------------------------------------------------------------------------------
// TMEM <-> registers.  Shape 32x32b: thread t of the warp reads/writes TMEM lane
// (32 * (warp % 4) + t); .xN moves N consecutive 32-bit columns.  The load helpers include the
// wait so the register results are usable when they return.
// ------------------------------------------------------------------------------------------
#define TOKMIX_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                     "=r"(r[i + 6]), "=r"(r[i + 7])
#define TOKMIX_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                     "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : TOKMIX_R8(0), TOKMIX_R8(8)
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : TOKMIX_R8(0), TOKMIX_R8(8), TOKMIX_R8(16), TOKMIX_R8(24)
      : "r"(taddr)
      : "memory");
}

// two back-to-back 32-column loads (r[0..31] from column a, r[32..63] from column b) with a single wait
__device__ __forceinline__ void tmem_ld32x2(uint32_t a, uint32_t b, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : TOKMIX_R8(0), TOKMIX_R8(8), TOKMIX_R8(16), TOKMIX_R8(24), TOKMIX_R8(32), TOKMIX_R8(40), TOKMIX_R8(48),
        TOKMIX_R8(56)
      : "r"(a), "r"(b)
      : "memory");
}

// columns [c, c+64) with a single wait
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) { tmem_ld32x2(taddr, taddr + 32u, r); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      TOKMIX_W8(0), TOKMIX_W8(8)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      TOKMIX_W8(0), TOKMIX_W8(8), TOKMIX_W8(16), TOKMIX_W8(24)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#undef TOKMIX_R8
#undef TOKMIX_W8

// ------------------------------------------------------------------------------------------
// small numeric helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (low 16 bits), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}

// hardware base-2 exponential (MUFU.EX2), flush-to-zero
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Blackwell's three-input maximum (one instruction for two comparisons)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace tokmix
