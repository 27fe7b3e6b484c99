// The bounded wait of the library, run on purpose until it gives up: one thread waits on an mbarrier that nothing
// ever arrives at, with the same helper the GEMM kernels use (mbar_wait_for), so a test can see a wait run out, the
// error bit reach the caller's device error word and the context stay usable, without faulting, trapping or
// hanging the GPU.
#include "common.cuh"
#include "psgd_b200.h"

namespace psgd {
namespace {

__global__ void __launch_bounds__(32) wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_for(&bar, 0, &abort, limit_ns)) atomicOr(err, ERR_TIMEOUT_FULL);
}

}  // namespace
}  // namespace psgd

extern "C" int psgd_wait_probe(int* dev_err, unsigned long long limit_ns, cudaStream_t stream) {
  using namespace psgd;
  if (!dev_err || limit_ns == 0 || limit_ns > WAIT_LIMIT_NS) return PSGD_EINVAL;
  wait_probe_kernel<<<1, 32, 0, stream>>>(dev_err, limit_ns);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}
