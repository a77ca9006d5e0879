// Activation helpers shared by the elementwise epilogues (sm_100a).
#pragma once

#include "f32x2.cuh"

namespace vh {

// gelu(x) = x/2 (1 + erf(x / sqrt 2)) for two lanes.  With a = |z|, t = 1 / (1 + p a),
// erfc(a) ~= t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-a^2)  (A&S 7.1.26), and
// 1 + erf(z) = 1 + sign(z) (1 - erfc(a)), so gelu = h + h sign(z) (1 - erfc(a)) with h = x/2.
// exp and the reciprocal use the hardware approximations directly (relative error near
// 2^-22, far inside the bf16 rounding every GELU output here receives).
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
__device__ __forceinline__ float2 gelu2(float2 x) {
    constexpr float kP = 0.3275911f, kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f,
                    kA4 = -1.453152027f, kA5 = 1.061405429f;
    constexpr float kLog2e = 1.4426950408889634f;
    const float2 z = fmul2(x, splat2(0.70710678118654752f));
    const float2 d = ffma2(make_float2(fabsf(z.x), fabsf(z.y)), splat2(kP), splat2(1.f));
    const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    float2 q = ffma2(t, splat2(kA5), splat2(kA4));
    q = ffma2(q, t, splat2(kA3));
    q = ffma2(q, t, splat2(kA2));
    q = ffma2(q, t, splat2(kA1));
    q = fmul2(q, t);
    const float2 arg = fmul2(fmul2(z, z), splat2(-kLog2e));
    const float2 c = fmul2(q, make_float2(ex2_approx(arg.x), ex2_approx(arg.y)));  // erfc(|z|)
    const float2 om = ffma2(c, splat2(-1.f), splat2(1.f));                           // 1 - erfc(|z|)
    const float2 sg = make_float2(copysignf(om.x, z.x), copysignf(om.y, z.y));
    const float2 h = fmul2(x, splat2(0.5f));
    return ffma2(h, sg, h);
}

}  // namespace vh
