// Failure-path self test: a bounded mbarrier wait that nothing completes.  Every pipelined kernel
// of the library waits on mbarriers with the same limit (mbar_wait, about two seconds of wall time)
// and, when it runs out, ORs WGKV_ERR_TIMEOUT into the caller's error word and returns instead of
// hanging.  This entry point runs that path on purpose -- no fault, no trap -- so tests can check
// that the status arrives and that the context stays usable afterwards.
#include "common.cuh"

namespace wgkv {
namespace {

__global__ void wait_limit_probe_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected, none ever made
    fence_barrier_init();
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0) && threadIdx.x == 0) set_error(err, WGKV_ERR_TIMEOUT);
}

}  // namespace
}  // namespace wgkv

extern "C" int wgkv_selftest_wait_limit(int* err, void* stream) {
  if (!err) return WGKV_EINVAL;
  wgkv::wait_limit_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
