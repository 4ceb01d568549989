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

// 2^x from a Cody-Waite split x = j + f (j = round(x), |f| <= 0.5) and a degree-3 minimax
// polynomial for 2^f fitted here (max relative error 1.0e-4, well below bf16 rounding of
// P); 2^j is added into the exponent field. Inputs are clamped at -120 (so -inf gives
// ~7.5e-37 rather than a wrapped exponent). Packed f32x2 arithmetic, two values at once.
ZWG_DEV float2 exp2_poly2(float2 x) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
    x.x = fmaxf(x.x, -120.f);
    x.y = fmaxf(x.y, -120.f);
    const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 r = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(r, make_float2(-1.f, -1.f), x);
    float2 p = __ffma2_rn(make_float2(0.05500858277f, 0.05500858277f), f,
                          make_float2(0.24221037328f, 0.24221037328f));
    p = __ffma2_rn(p, f, make_float2(0.69328290224f, 0.69328290224f));
    p = __ffma2_rn(p, f, make_float2(1.f, 1.f));
    // the low bits of t hold j; shifting them into the exponent field scales by 2^j
    p.x = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
    p.y = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
    return p;
}

// max of three floats in one instruction (PTX three-input max.f32, sm_100a); a NaN operand
// is ignored as by fmaxf
ZWG_DEV float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
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
