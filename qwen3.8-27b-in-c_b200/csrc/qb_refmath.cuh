// Element-wise functions restated from the reference so that results match
// its values: the AVX2 polynomial exp (src/kernels.c:807-822) and the silu /
// sigmoid built on it (src/kernels.c:825-871).  Products the reference rounds
// separately (ISO C, no FP contraction) use the _rn intrinsics.
#pragma once
#include "qb_common.cuh"

namespace {

// AVX2 exp of the reference (src/kernels.c:807-822), lane-for-lane.
__device__ __forceinline__ float exp_poly(float x) {
    const float xc = fmaxf(fminf(x, 88.0f), -88.0f);
    const float k = rintf(__fmul_rn(xc, 1.4426950408889634f));
    const float r = fmaf(-k, 0.6931471805599453f, xc);
    float p = 0.000198412698f;
    p = fmaf(p, r, 0.00139304842f);
    p = fmaf(p, r, 0.00833333333f);
    p = fmaf(p, r, 0.04166666666f);
    p = fmaf(p, r, 0.16666666666f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ik = (int)k;
    const float pow2 = __int_as_float((int)((unsigned)(ik + 127) << 23));
    return __fmul_rn(p, pow2);
}

// silu / sigmoid of the vector body (src/kernels.c:825-871); the reference
// only takes its scalar tail for n % 8 != 0, which no layer width hits.
__device__ __forceinline__ float silu_ref(float v) {
    const float e = exp_poly(__fsub_rn(0.0f, v));
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(v, sig);
}
__device__ __forceinline__ float sigmoid_ref(float v) {
    const float e = exp_poly(__fsub_rn(0.0f, v));
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}
}  // namespace
