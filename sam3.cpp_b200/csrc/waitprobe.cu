// Self-test of the bounded device waits every kernel of the engine uses (mbar_wait, common.cuh).
//
// One CTA initialises an mbarrier that expects one arrive, optionally withholds that arrive, and waits
// on it with mbar_wait_for and a caller-chosen limit. When the arrive is withheld nothing can complete
// the phase, so the wait must give up after the limit, record kErrWaitMisc in the error word and let the
// kernel return: the same path a GEMM or attention kernel takes when a TMA stage or an accumulator never
// arrives, exercised without faulting or hanging the GPU.
#include "common.cuh"
#include "kernels.h"

namespace s3b {

namespace {

__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns, int withhold) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!withhold) mbar_arrive(&bar);
    mbar_wait_for(&bar, 0, &abort_flag, err, kErrWaitMisc, limit_ns);
  }
  __syncthreads();
}

}  // namespace

int wait_probe(int* err, long long limit_ns, int withhold, cudaStream_t st) {
  if (!err || limit_ns <= 0 || limit_ns > (long long)kWaitNs) return -2;
  wait_probe_kernel<<<1, 32, 0, st>>>(err, (unsigned long long)limit_ns, withhold ? 1 : 0);
  return launch_status("wait_probe");
}

}  // namespace s3b
