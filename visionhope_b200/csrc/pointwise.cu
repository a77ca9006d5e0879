// Bias (+ exact GELU) over channels-last rows: the epilogue of a convolution whose
// BatchNorm has been folded into it (stem and downsample layers, models/layers.py:85-107).
// y = act(x + b[c]) computed in fp32 and rounded once to y's dtype; 8-channel vectors.
// Residual add with a cast: y = (y dtype)(x + r), the stage's last residual add
// (models/block.py:106) fused with the autocast cast of the downsample convolution's input.
#include <algorithm>

#include "abi_util.h"
#include "activations.cuh"
#include "common.cuh"

namespace vh {
namespace {

constexpr int kPwThreads = 256;

template <typename XT, typename YT, bool GELU>
__global__ void __launch_bounds__(kPwThreads) bias_act_kernel(const XT* __restrict__ x, const float* __restrict__ bias,
                                                              YT* __restrict__ y, int64_t groups, int C) {
    const int G = C / 8;
    for (int64_t i = blockIdx.x * (int64_t)kPwThreads + threadIdx.x; i < groups; i += (int64_t)gridDim.x * kPwThreads) {
        const int c = (int)(i % G) * 8;
        float v[8], b[8];
        load8(x + i * 8, v);
        load8(bias + c, b);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            float2 t = fadd2(make_float2(v[e], v[e + 1]), make_float2(b[e], b[e + 1]));
            if (GELU) t = gelu2(t);
            v[e] = t.x;
            v[e + 1] = t.y;
        }
        store8(y + i * 8, v);
    }
}

template <typename XT, typename YT>
int bias_act_run(const void* x, const float* bias, void* y, int64_t rows, int C, int act, cudaStream_t st) {
    const int64_t groups = rows * (C / 8);
    const int grid = (int)std::min<int64_t>((groups + kPwThreads - 1) / kPwThreads, (int64_t)sm_count() * 16);
    if (act == VH_ACT_GELU)
        bias_act_kernel<XT, YT, true><<<grid, kPwThreads, 0, st>>>(static_cast<const XT*>(x), bias, static_cast<YT*>(y), groups, C);
    else
        bias_act_kernel<XT, YT, false><<<grid, kPwThreads, 0, st>>>(static_cast<const XT*>(x), bias, static_cast<YT*>(y), groups, C);
    return launch_status("bias act");
}

template <typename XT>
int bias_act_y(int y_dtype, const void* x, const float* bias, void* y, int64_t rows, int C, int act, cudaStream_t st) {
    switch (y_dtype) {
        case VH_F32: return bias_act_run<XT, float>(x, bias, y, rows, C, act, st);
        case VH_BF16: return bias_act_run<XT, __nv_bfloat16>(x, bias, y, rows, C, act, st);
        default: return bias_act_run<XT, __half>(x, bias, y, rows, C, act, st);
    }
}

constexpr int kAddUnroll = 4;

template <typename XT, typename RT, typename YT>
__global__ void __launch_bounds__(kPwThreads) add_cast_kernel(const XT* __restrict__ x, const RT* __restrict__ r,
                                                              YT* __restrict__ y, int64_t groups) {
    const int64_t stride = (int64_t)gridDim.x * kPwThreads;
    for (int64_t i0 = blockIdx.x * (int64_t)kPwThreads + threadIdx.x; i0 < groups; i0 += stride * kAddUnroll) {
        float v[kAddUnroll][8], a[kAddUnroll][8];
#pragma unroll
        for (int u = 0; u < kAddUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < groups) {
                load8(x + i * 8, v[u]);
                load8(r + i * 8, a[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < kAddUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            if (i >= groups) break;
#pragma unroll
            for (int e = 0; e < 8; ++e) v[u][e] += a[u][e];
            store8(y + i * 8, v[u]);
        }
    }
}

template <typename XT, typename RT, typename YT>
int add_cast_run(const void* x, const void* r, void* y, int64_t n, cudaStream_t st) {
    const int64_t groups = n / 8;
    const int grid = (int)std::min<int64_t>((groups + kPwThreads - 1) / kPwThreads, (int64_t)sm_count() * 8);
    add_cast_kernel<XT, RT, YT><<<grid, kPwThreads, 0, st>>>(static_cast<const XT*>(x), static_cast<const RT*>(r),
                                                             static_cast<YT*>(y), groups);
    return launch_status("add cast");
}

template <typename XT, typename RT>
int add_cast_y(int y_dtype, const void* x, const void* r, void* y, int64_t n, cudaStream_t st) {
    return y_dtype == VH_F32 ? add_cast_run<XT, RT, float>(x, r, y, n, st)
                             : add_cast_run<XT, RT, __nv_bfloat16>(x, r, y, n, st);
}

}  // namespace
}  // namespace vh

using namespace vh;

extern "C" int vh_add_cast_fwd(const void* x, int32_t x_dtype, const void* r, int32_t r_dtype, void* y,
                               int32_t y_dtype, int64_t n, vh_stream_t stream) {
    clear_error();
    if (!x || !r || !y) return fail(VH_E_ARG, "vh_add_cast_fwd: null pointer argument");
    auto ok = [](int d) { return d == VH_F32 || d == VH_BF16; };
    if (!ok(x_dtype) || !ok(r_dtype) || !ok(y_dtype)) return fail(VH_E_DTYPE, "vh_add_cast_fwd: dtypes must be fp32 or bf16");
    if (n <= 0 || n % 8) return fail(VH_E_SHAPE, "vh_add_cast_fwd: the element count must be a positive multiple of 8");
    if (!aligned(x, 16) || !aligned(r, 16) || !aligned(y, 16))
        return fail(VH_E_ALIGN, "vh_add_cast_fwd: x, r and y must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (x_dtype == VH_F32)
        return r_dtype == VH_F32 ? add_cast_y<float, float>(y_dtype, x, r, y, n, st)
                                 : add_cast_y<float, __nv_bfloat16>(y_dtype, x, r, y, n, st);
    return r_dtype == VH_F32 ? add_cast_y<__nv_bfloat16, float>(y_dtype, x, r, y, n, st)
                             : add_cast_y<__nv_bfloat16, __nv_bfloat16>(y_dtype, x, r, y, n, st);
}

extern "C" int vh_bias_act_fwd(const void* x, int32_t x_dtype, const float* bias, void* y, int32_t y_dtype,
                               int64_t rows, int32_t channels, int32_t act, vh_stream_t stream) {
    clear_error();
    if (!x || !bias || !y) return fail(VH_E_ARG, "vh_bias_act_fwd: null pointer argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(VH_E_DTYPE, "vh_bias_act_fwd: bad dtype");
    if (act != VH_ACT_NONE && act != VH_ACT_GELU) return fail(VH_E_ARG, "vh_bias_act_fwd: bad activation %d", act);
    if (rows <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_bias_act_fwd: empty input");
    if (channels % 8) return fail(VH_E_SHAPE, "vh_bias_act_fwd: channels must be a multiple of 8");
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(bias, 16))
        return fail(VH_E_ALIGN, "vh_bias_act_fwd: x, y and bias must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case VH_F32: return bias_act_y<float>(y_dtype, x, bias, y, rows, channels, act, st);
        case VH_BF16: return bias_act_y<__nv_bfloat16>(y_dtype, x, bias, y, rows, channels, act, st);
        default: return bias_act_y<__half>(y_dtype, x, bias, y, rows, channels, act, st);
    }
}
