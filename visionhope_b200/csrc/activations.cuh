// Activation helpers shared by the elementwise epilogues (sm_100a).
#pragma once

#include "f32x2.cuh"

namespace vh {

// The hardware approximations of 2^v and 1/v (flush-to-zero).
__device__ __forceinline__ float ex2_approx(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
__device__ __forceinline__ float rcp_approx(float v) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
// gelu(x) = x Phi(x) for two lanes, Phi(x) = (1 + erf(x / sqrt 2)) / 2.  With a = |x| / sqrt 2,
// t = 1 / (1 + p a) and erfc(a) ~= t P(t) exp(-a^2), P(t) = a1 + a2 t + ... + a5 t^4
// (Abramowitz & Stegun 7.1.26, |error| <= 1.5e-7):
//   Phi(x) = 1/2 + sign(x) (1/2 - erfc(a) / 2),  so  gelu(x) = x/2 + |x| m,
//   m = 1/2 + Q exp(-a^2),  Q = t P'(t),  P' = -P / 2,
// with 1/sqrt 2 folded into p and the exponent's scale.  exp and the reciprocal use the
// hardware approximations (relative error near 2^-22, far inside the bf16 rounding every GELU
// output here receives).
__device__ __forceinline__ float2 gelu2(float2 x) {
    constexpr float kP = 0.3275911f * 0.70710678118654752f;
    constexpr float kA1 = -0.5f * 0.254829592f, kA2 = -0.5f * -0.284496736f, kA3 = -0.5f * 1.421413741f,
                    kA4 = -0.5f * -1.453152027f, kA5 = -0.5f * 1.061405429f;
    constexpr float kE = -0.5f * 1.4426950408889634f;  // exp(-x^2 / 2) = 2^(kE x^2)
    const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 d = ffma2(ax, splat2(kP), splat2(1.f));
    const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    float2 q = ffma2(t, splat2(kA5), splat2(kA4));
    q = ffma2(q, t, splat2(kA3));
    q = ffma2(q, t, splat2(kA2));
    q = ffma2(q, t, splat2(kA1));
    q = fmul2(q, t);
    const float2 arg = fmul2(fmul2(x, x), splat2(kE));
    const float2 m = ffma2(q, make_float2(ex2_approx(arg.x), ex2_approx(arg.y)), splat2(0.5f));
    return ffma2(ax, m, fmul2(x, splat2(0.5f)));
}

}  // namespace vh
