// selftest.cu -- a device-side check of the bounded waits that every pipelined kernel of this
// library relies on to end instead of hanging the GPU.
//
// The kernels' waits (mbar_wait, wait_flag in sm100.cuh) give up after kWaitTimeoutNs, set a
// TOKMIX_DEV_* bit in the caller's device status word, raise the CTA's abort flag so that the
// other warps stop waiting too, and return false.  This entry point runs those same functions on
// a wait that nothing will ever satisfy, with a short limit, so that a test can watch the whole
// path -- the limit running out, the status bit, the second warp draining on the abort flag, the
// host-side error -- without a fault: nothing is in flight (no TMA copy, no MMA, no TMEM).
#include <cuda_runtime.h>

#include "host_common.h"
#include "sm100.cuh"

namespace tokmix {
namespace selftest {

// which = 0: a transaction barrier expecting bytes that never arrive (a TMA load that never lands)
// which = 1: a hand-off barrier expecting two arrivals that receives one
// which = 2: a ready flag in global memory (`flag`) that nobody sets -- or, if the caller set it,
//            a wait that succeeds
// Warp 0 lane 0 waits with `limit_ns`; warp 1 lane 0 waits on the same event with the library's
// own limit and must return as soon as warp 0 has given up.  result[w] = what warp w's wait
// returned (1 = satisfied, 0 = gave up).
__global__ void wait_timeout_kernel(int which, unsigned long long limit_ns, const uint32_t* flag, int32_t* result,
                                    uint32_t* status) {
  __shared__ uint64_t bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    cta_abort_flag() = 0u;
    mbar_init(&bar, which == 1 ? 2u : 1u);
    fence_barrier_init();
    if (which == 0) mbar_arrive_expect_tx(&bar, 1024u);  // completes only once 1024 bytes land
    if (which == 1) mbar_arrive(&bar);                   // the second arrival never comes
  }
  __syncthreads();
  if (lane == 0) {
    const unsigned long long lim = warp == 0 ? limit_ns : kWaitTimeoutNs;
    bool ok;
    if (which == 2) {
      ok = wait_flag(flag, status, lim);
    } else {
      ok = mbar_wait(&bar, 0, status, which == 0 ? kDevTimeoutTma : kDevTimeoutPipe, lim);
    }
    if (result != nullptr) result[warp] = ok ? 1 : 0;
  }
}

}  // namespace selftest
}  // namespace tokmix

extern "C" int tokmix_selftest_wait_timeout(int which, long long limit_ns, const uint32_t* flag, int32_t* result,
                                            uint32_t* status, void* stream) {
  using namespace tokmix;
  if (which < 0 || which > 2) return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_selftest_wait_timeout: which must be 0, 1 or 2");
  if (limit_ns < 1000 || limit_ns > 1000000000ll)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_selftest_wait_timeout: limit_ns must be in [1e3, 1e9]");
  if (status == nullptr || (which == 2 && flag == nullptr))
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_selftest_wait_timeout: null status word or flag");
  if (reinterpret_cast<uintptr_t>(status) % 4 != 0 || reinterpret_cast<uintptr_t>(flag) % 4 != 0 ||
      reinterpret_cast<uintptr_t>(result) % 4 != 0)
    return fail(TOKMIX_ERR_INVALID_ARGUMENT, "tokmix_selftest_wait_timeout: pointers must be 4-byte aligned");
  if (const int rc = check_device()) return rc;
  selftest::wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      which, static_cast<unsigned long long>(limit_ns), flag, result, status);
  return check_launch("tokmix_selftest_wait_timeout");
}
