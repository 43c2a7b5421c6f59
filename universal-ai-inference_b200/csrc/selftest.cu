// selftest.cu -- exercises the bounded-wait failure path of the tensor-core
// kernels on the device without faulting anything: the threads of one block
// wait on an mbarrier that nothing ever arrives on, through the same
// bounded_wait the expert kernel uses, with a short budget.  Each gives up,
// the first records its code in the backend's device error word, and the
// kernel returns normally; the host then reports the error status and the
// context stays usable.
#include "kernels.hpp"
#include "umma.cuh"

namespace uaii_b200 {
namespace {

__global__ void wait_timeout_selftest_kernel(int* err, long long budget, int code) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    umma::mbar_init(&bar, 1);
    umma::fence_barrier_init();
    abort_flag = 0;
  }
  __syncthreads();
  // phase 0 of `bar` never completes: every thread must give up within the budget
  (void)umma::bounded_wait(&bar, 0, &abort_flag, err, code, budget);
  __syncthreads();
}

}  // namespace

cudaError_t launch_wait_timeout_selftest(int* err, long long budget_cycles, int code, cudaStream_t st) {
  if (budget_cycles < 1000 || budget_cycles > 4000000000LL) return cudaErrorInvalidValue;
  wait_timeout_selftest_kernel<<<1, 64, 0, st>>>(err, budget_cycles, code);
  return cudaGetLastError();
}

}  // namespace uaii_b200
