// Self-test of the device-side failure detection.  Every wait of the
// pipelined kernels is bounded: when the event it waits for never comes, the
// wait gives up after its time limit, records an error bit and the waiting
// site, and the kernel returns, so the context stays usable.  This kernel
// exercises exactly that path: one thread waits on an mbarrier that nothing
// completes.  No reference counterpart.
#include "spk_common.cuh"

namespace spk {

__global__ void selftest_wait_kernel() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait(&bar, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);  // phase 0 never completes: gives up after the bound
  }
}

}  // namespace spk

extern "C" int spk_selftest_wait_timeout(spk_stream_t stream) {
  spk::selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>();
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}
