// Self-test of the device-side failure detection.
//
// Every kernel of the library waits on mbarriers through mbar_wait (ptx.cuh):
// a wait that runs past its limit records an error code in the caller's
// status word and returns false, and the kernel skips its remaining work.  The
// kernel here exercises exactly that path on a barrier that, when asked,
// nobody ever arrives on, with a short caller-chosen limit, so the host side
// (mea_read_status, the Python binding) can be tested against a real device
// timeout without a fault or a hang: the wait always ends by its limit.
#include "launch.h"
#include "ptx.cuh"

namespace mea {

// One warp.  Thread 0 initialises an mbarrier expecting one arrival; with
// `arrive` set the same thread arrives at once (the wait completes), otherwise
// no thread does and the bounded wait of every lane gives up after limit_ns.
__global__ void __launch_bounds__(32) selftest_wait_kernel(int* status, unsigned long long limit_ns, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) mbar_arrive(b);
  __syncwarp();
  Guard g(status, KID_TEST);
  mbar_wait_for(b, 0, g, 1, limit_ns);
}

}  // namespace mea

extern "C" int mea_selftest_wait(int* status, unsigned long long limit_ns, int arrive, void* stream) {
  using namespace mea;
  if (!status) return set_error(MEA_ERR_INVALID_ARGUMENT, "selftest: status is NULL");
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "selftest: limit_ns must be in (0, 1e9]");
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns, arrive);
  return check_launch("selftest_wait_kernel");
}
