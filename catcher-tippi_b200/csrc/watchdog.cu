// Device watchdog check: one kernel waits, through the library's bounded
// mbarrier wait (common.cuh, the wait every TMA pipeline here uses), on a
// barrier that nothing ever arrives on.  The wait gives up after its limit
// (2 s), sets the timeout bit of the device status word and returns, and the
// kernel ends normally -- the path a real stalled copy would take, exercised
// without a fault, a trap or an unbounded loop, so the context stays usable.
#include <string>

#include "capi_guard.hpp"
#include "common.cuh"
#include "device_buffer.hpp"
#include "qlinear.hpp"

namespace {

__global__ void watchdog_probe_kernel(int* status, int* outcome) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    cq::mbar_init(&bar, 1);  // one arrival expected; none will come
    cq::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool arrived = cq::mbar_wait_bounded(&bar, 0, status);
    *outcome = arrived ? 1 : 2;  // 2: the wait gave up and the kernel went on
  }
}

}  // namespace

extern "C" cq_status cq_device_watchdog_check(int32_t device) {
  using namespace nemotron_cuda;
  return guarded([&] {
    DeviceContext& ctx = device_context(device);
    DeviceGuard guard(device);
    DeviceBuffer outcome(sizeof(int));
    check_cuda(cudaMemset(outcome.get(), 0, sizeof(int)), "clear outcome");
    watchdog_probe_kernel<<<1, 32>>>(ctx.status, outcome.as<int>());
    check_cuda(cudaGetLastError(), "watchdog probe launch");
    check_cuda(cudaDeviceSynchronize(), "watchdog probe");
    int got = 0, status = 0;
    check_cuda(cudaMemcpy(&got, outcome.get(), sizeof(int), cudaMemcpyDeviceToHost), "read outcome");
    check_cuda(cudaMemcpy(&status, ctx.status, sizeof(int), cudaMemcpyDeviceToHost), "read status");
    if (got != 2 || (status & cq::kStatusWaitTimeout) == 0)
      throw Error(CQ_RUNTIME_ERROR, "device watchdog check failed: outcome " + std::to_string(got) +
                                        ", status " + std::to_string(status));
  });
}
