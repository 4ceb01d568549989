// Self-test of the device-side timeout path: one bounded mbarrier wait that nothing
// completes. Every kernel of the library waits through sm100::mbar_wait, which gives up
// after a few seconds, records kErrTimeout in the context's error word and returns, so a
// lost arrival (a failed copy, a bug) ends the call with ZWG_TIMEOUT instead of a hung GPU.
// This kernel runs exactly that wait on a barrier no thread or copy ever arrives on, so a
// caller (or a test) can see the whole path work: the wait runs out, the kernel returns,
// the host reads ZWG_TIMEOUT, and the context stays usable.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace zwg {

__global__ void wait_timeout_selftest_kernel(int* err, int* gave_up) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);  // one arrival expected; none is ever made
        sm100::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) *gave_up = sm100::mbar_wait(&bar, 0, err) ? 0 : 1;
}

int wait_timeout_selftest_launch(int* err, int* gave_up, cudaStream_t st) {
    wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(err, gave_up);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace zwg
