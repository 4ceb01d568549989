// Programmatic dependent launch for chains of short kernels (the projections, norms and
// sampling around the attention calls of a decode step).
//
// A kernel launched through launch_chained may start while the kernel before it on the
// stream is still running. It must call chain_release() to let the next kernel start
// early and chain_wait() before it reads anything an earlier kernel wrote or writes
// anything an earlier kernel reads; work on constants (weight prefetch) may come before
// the wait. Kernels not launched this way are unaffected: the wait returns at once, and a
// kernel launched the ordinary way after a chained one waits for it to complete.
//
// chain_wait() returns 0 through an asm output the compiler cannot see through. Kernels
// add it to every data pointer they use after the wait, so no load can be scheduled
// above the wait. The wait makes the previous grids' writes visible to this grid, so data
// they wrote is read after it with ordinary (coherent, L1-cached) loads; the
// non-coherent read-only path (__ldg) is kept for constants such as the weights.
#pragma once
#include <cuda_runtime.h>

namespace zwg {

__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ int chain_wait() {
    int z;
    asm volatile("griddepcontrol.wait;\n\tmov.u32 %0, 0;" : "=r"(z) : : "memory");
    return z;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_chained_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_chained(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    return launch_chained_smem(kern, grid, block, 0, st, args...);
}

}  // namespace zwg
