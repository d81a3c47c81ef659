// Self-test of the bounded mbarrier wait (the failure path of the tensor-core
// kernels), runnable without faulting or hanging the GPU.
//
// One warp initialises an mbarrier that expects one arrival; nobody arrives,
// so its phase 0 never completes, and lane 0 waits on it through the same
// loop the grouped GEMM and the router use (mbar_wait_until), with a short
// limit instead of their 2 s.  The wait must give up, set the CTA's abort
// flag, record {1 (timeout), kSelftestSite, block 0} in the status word and
// return, after which the kernel exits normally and the context stays usable.
#include "kernels.h"
#include "tc.cuh"

namespace parrot {

namespace {

__global__ void __launch_bounds__(32) mbar_timeout_selftest_kernel(unsigned long long limit_ns,
                                                                   int* out) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_timer_ns();
    const bool ok = tc::mbar_wait_until(&bar, 0, &abort_flag, out, kSelftestSite, limit_ns);
    const uint64_t waited = global_timer_ns() - t0;
    out[4] = ok ? 1 : 0;
    out[5] = abort_flag;
    const uint64_t us = waited / 1000;
    out[6] = us > 0x7fffffffull ? 0x7fffffff : (int)us;  // microseconds
  }
}

}  // namespace

int launch_mbar_timeout_selftest(unsigned long long limit_ns, int* out, cudaStream_t stream) {
  mbar_timeout_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace parrot
