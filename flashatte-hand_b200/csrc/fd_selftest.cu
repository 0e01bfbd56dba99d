// fd_selftest.cu - exercises the bounded mbarrier wait the decode kernel uses
// for every pipeline hand-off: a wait on a barrier that nothing will ever
// arrive on must give up after its time budget, report it, and leave the
// context usable.  No memory fault, trap or endless loop is involved.
#include "fd_kernels.h"
#include "fd_ptx.cuh"

namespace fd {

namespace {

__global__ void bounded_wait_probe_kernel(unsigned long long budget_ns, int* status,
                                          unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival; none is ever made
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    const bool ok = mbar_wait_bounded(&bar, 0, &abort_flag, budget_ns);
    *waited_ns = globaltimer_ns() - t0;
    *status = ok ? 0 : 5;
  }
}

}  // namespace

cudaError_t launch_bounded_wait_probe(unsigned long long budget_ns, int* status,
                                      unsigned long long* waited_ns, cudaStream_t stream) {
  bounded_wait_probe_kernel<<<1, 32, 0, stream>>>(budget_ns, status, waited_ns);
  return cudaGetLastError();
}

}  // namespace fd
