// Self-test of the device-side failure path: a kernel whose bounded wait runs out.
//
// Every kernel of this library waits on mbarriers only through mbar_wait / mbar_wait_for (common.cuh):
// a wait that does not complete within its limit sets the CTA's abort flag, records (site, block, thread)
// in the device error record and returns false, and the kernel unwinds (freeing its tensor memory) instead
// of spinning forever or trapping.  This entry point runs exactly that path on purpose, without any fault:
// one CTA of four warps allocates tensor memory like the production kernels, then every warp waits on an
// mbarrier phase that nothing ever completes, with the caller's short limit.  The first waiter to give up
// records the error and raises the abort flag; the others see the flag and leave; warp 0 frees the tensor
// memory and the kernel returns.  bf_device_error then reports the timeout, and the context stays usable.
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr unsigned int kSelftestSite = 0xF1;

__global__ void __launch_bounds__(128, 1) selftest_wait_kernel(uint64_t limit_ns, unsigned int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // one arrival completes the phase; nothing arrives
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // lane 0 of every warp waits (as the producer / MMA warps do); the warp follows its lane 0
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_for(&bar, 0, &abort_flag, err, kSelftestSite, limit_ns);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  (void)ok;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 32);
}

}  // namespace bfb

using namespace bfb;

extern "C" int bf_selftest_wait_timeout(unsigned int limit_us, bf_stream_t stream) {
  if (limit_us == 0 || limit_us > 1000000u) return BF_ERR_INVALID_ARGUMENT;
  DeviceState st;
  const int rc = device_state(&st);
  if (rc) return rc;
  selftest_wait_kernel<<<1, 128, 0, stream>>>((uint64_t)limit_us * 1000ull, st.err);
  return launch_status();
}
