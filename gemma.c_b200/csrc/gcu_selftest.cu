// gcu_selftest.cu -- failure-detection self-test of the device-side waits.
//
// Every wait in the library's kernels (TMA stages, accumulator hand-offs,
// split-K partials, peer ranks of the fused all-gather) is bounded by a
// %globaltimer budget: on expiry the kernel records a code in the device
// error word and returns, and the host reports "device-side wait gave up"
// at its next check.  This entry point runs one of those waits on something
// that never completes -- a shared-memory mbarrier nobody arrives on (the
// TMA/MMA pipeline's wait) or a global flag nobody sets (the split-K and
// peer-rank wait) -- with a short budget, so a test can show that the wait
// ends, the host sees the code, and the context keeps working.  No fault,
// trap or endless loop is involved.
#include "gcu_internal.cuh"

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

__device__ int g_never_set;  // zero-initialised, written by nothing
__device__ unsigned long long g_waited_ns;

__global__ void k_wait_selftest(int mode, unsigned int *err, unsigned long long budget_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint64_t t0 = ptx::globaltimer();
  if (mode == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_wait(&bar, 0, err, DEV_TIMEOUT_SELFTEST, budget_ns);  // phase 0 never completes
  } else {
    ptx::flag_wait_geq<true>(&g_never_set, 1, t0, err, DEV_TIMEOUT_SELFTEST, budget_ns);
  }
  g_waited_ns = ptx::globaltimer() - t0;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

// mode 0: mbarrier wait, 1: flag wait.  budget_us in [1, 1000000].  On
// return (the stream synchronised) the error word holds DEV_TIMEOUT_SELFTEST
// and *waited_ns, if given, the kernel's own measure of the wait.
GCU_EXPORT int gcu_selftest_bounded_wait(int mode, int budget_us, unsigned long long *waited_ns,
                                         void *stream) {
  if (mode != 0 && mode != 1) return set_error("selftest_bounded_wait: mode %d is not 0 or 1", mode);
  if (budget_us < 1 || budget_us > 1000000)
    return set_error("selftest_bounded_wait: budget %d us outside [1, 1000000]", budget_us);
  unsigned int *ew = dev_error_word();
  if (!ew) return set_error("selftest_bounded_wait: no device error word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_wait_selftest<<<1, 32, 0, st>>>(mode, ew, 1000ull * (unsigned long long)budget_us);
  GCU_CUDA(cudaGetLastError());
  GCU_CUDA(cudaStreamSynchronize(st));
  if (waited_ns) GCU_CUDA(cudaMemcpyFromSymbol(waited_ns, g_waited_ns, sizeof(*waited_ns)));
  return 0;
}
