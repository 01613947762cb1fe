// sf_selftest_wait: exercises the bounded device-side wait that every tcgen05
// kernel of this library uses, without faulting or hanging anything.
//
// One warp initialises an mbarrier that expects a single arrival; with
// `arrive` != 0 lane 0 arrives on it, otherwise nothing ever does.  Every lane
// then waits on phase 0 through tc::mbar_wait with a bound of `polls` polls.
// A wait that runs out records SF_ERR_TIMEOUT in the library's per-device
// status word (the first error wins) and the kernel returns normally, which is
// what a production kernel does when one of its barriers is never completed.
// A second wait on the same barrier then polls only once (the thread is
// "aborted"), as the abort path of the production kernels relies on.
#include "sf_tc.cuh"

namespace sf {
namespace {

__global__ void __launch_bounds__(32) k_wait_selftest(uint32_t polls, int arrive, uint32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) tc::mbar_arrive(&bar);
  bool aborted = false;
  if (!tc::mbar_wait(&bar, 0, status, aborted, polls)) tc::mbar_wait(&bar, 0, status, aborted, polls);
  __syncwarp();
}

}  // namespace
}  // namespace sf

extern "C" int sf_selftest_wait(uint32_t polls, int arrive, sf_stream_t stream) {
  SF_REQUIRE(polls >= 1 && polls <= sf::tc::kWaitLimit, "sf_selftest_wait: polls must be in [1, %u]",
             sf::tc::kWaitLimit);
  uint32_t* status = sf::device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  sf::k_wait_selftest<<<1, 32, 0, stream>>>(polls, arrive, status);
  sf::count_launch();
  return sf::check_launch("sf_selftest_wait");
}
