// Shared device helpers for the zwgpu kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define ZWG_DEV __device__ __forceinline__

namespace zwg {

// Device-side error word codes, written by kernels and read by the host after a sync.
enum : int {
    kErrNone = 0,
    kErrTimeout = 1,   // a bounded wait ran out
    kErrBounds = 2,    // a checked index was out of range (ZWG_CHECK builds)
};

// Iteration limit for every spin-wait on an mbarrier. With the back-off below this is
// several seconds, far above any legitimate wait in these kernels.
constexpr uint32_t kSpinLimit = 1u << 26;

ZWG_DEV void set_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Online-softmax helpers -----------------------------------------------------------------

// exp(x) for x <= 0 through the hardware base-2 exponential: callers pass scores already
// multiplied by log2(e), so one ex2.approx is the whole exponential.
ZWG_DEV float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

ZWG_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

ZWG_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace zwg
