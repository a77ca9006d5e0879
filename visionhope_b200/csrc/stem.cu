// First layer of the VisionHOPE stem (models/layers.py:85-107): 3x3 convolution, stride 2,
// padding 1, of the 3-channel input image, with its BatchNorm folded in and the bias + GELU
// epilogue, as one kernel.
//
// A library convolution spends most of its time on a 3-channel input: the input is padded to
// a wider channel count and cast to bf16 in separate passes, and the bias + GELU runs after it
// as one more pass over the output.  Here the 27-long reduction of every output pixel is an
// implicit GEMM on tensor cores: a warp owns 16 output pixels at a time (the MMA rows) and the
// 27 taps x channels, padded to 32, are the MMA's K.  A CTA stages its input window (rows
// 2*TH+1, columns 2*TW+1, 3 channels) in shared memory rounded to bf16, with zeros outside the
// image; each lane gathers its A-fragment elements from there through per-lane tap offsets.
// The weights (bf16, as autocast feeds them) sit in registers as B fragments for the whole CTA.
//
// Arithmetic follows the model's path under bf16 autocast: x and w rounded to bf16, fp32
// accumulation, the convolution's output rounded to bf16, then fp32 bias, exact-erf GELU
// (Abramowitz & Stegun 7.1.26) and one rounding to the output dtype.
#include <algorithm>

#include "abi_util.h"
#include "activations.cuh"
#include "common.cuh"
#include "srnl_scan.cuh"

namespace vh {
namespace {

constexpr int kStemWarps = 4;
constexpr int kStemRowsPerWarp = 4;      // output rows of the tile per warp
constexpr int kStemTW = 32;              // output columns per tile (two 16-pixel MMA tiles)
constexpr int kStemTH = kStemWarps * kStemRowsPerWarp;  // output rows per tile
constexpr int kStemIH = 2 * kStemTH + 1; // staged input rows
constexpr int kStemIW = 2 * kStemTW + 1; // staged input columns
constexpr int kStemCin = 3;

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

template <int NT, bool GELU, typename YT>
__global__ void __launch_bounds__(32 * kStemWarps) stem_conv_kernel(const float* __restrict__ x,
                                                                    const float* __restrict__ w,
                                                                    const float* __restrict__ bias,
                                                                    YT* __restrict__ y, int H, int W, int Ho,
                                                                    int Wo, int tiles_w) {
    constexpr int COUT = 8 * NT;
    __shared__ __nv_bfloat16 xs[kStemIH * kStemIW * kStemCin];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qg = lane >> 2, qt = lane & 3;
    const int b = blockIdx.y;
    const int oy0 = (blockIdx.x / tiles_w) * kStemTH, ox0 = (blockIdx.x % tiles_w) * kStemTW;
    const int iy0 = 2 * oy0 - 1, ix0 = 2 * ox0 - 1;

    // Input window, rounded to bf16, zeros outside the image (the convolution's padding);
    // the loads of a batch are issued before any is converted.
    const float* xb = x + (int64_t)b * H * W * kStemCin;
    constexpr int kN = kStemIH * kStemIW * kStemCin, kT = 32 * kStemWarps, kBatch = 8;
    for (int i0 = tid; i0 < kN; i0 += kT * kBatch) {
        float v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = i0 + u * kT;
            const int c = i % kStemCin, pix = i / kStemCin;
            const int gy = iy0 + pix / kStemIW, gx = ix0 + pix % kStemIW;
            v[u] = 0.f;
            if (i < kN && gy >= 0 && gy < H && gx >= 0 && gx < W) v[u] = __ldg(xb + ((int64_t)gy * W + gx) * kStemCin + c);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            if (i0 + u * kT < kN) xs[i0 + u * kT] = __float2bfloat16_rn(v[u]);
    }

    // B fragments: B[k][n] = w[n][c][ky][kx] with k = (ky * 3 + kx) * 3 + c (k >= 27: zero).
    uint32_t bf[NT][2][2];
    // Shared-memory offsets (elements) of this lane's A columns k, relative to the pixel's
    // window origin; -1 marks the padded columns.
    int koff[2][4];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = 16 * s + 2 * qt + (j & 1) + 8 * (j >> 1);
            const int tap = k / 3, c = k % 3, ky = tap / 3, kx = tap % 3;
            koff[s][j] = k < 27 ? (ky * kStemIW + kx) * kStemCin + c : -1;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int n = 8 * t + qg;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                __nv_bfloat16 e[2];
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    const int k = 16 * s + 8 * h + 2 * qt + l;
                    const int tap = k / 3, c = k % 3;
                    e[l] = __float2bfloat16_rn(k < 27 ? w[(n * kStemCin + c) * 9 + tap] : 0.f);
                }
                bf[t][s][h] = pack_bf16x2(e[0], e[1]);
            }
        }
    }
    float bv[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        bv[t][0] = bias[8 * t + 2 * qt];
        bv[t][1] = bias[8 * t + 2 * qt + 1];
    }
    __syncthreads();

    for (int rr = 0; rr < kStemRowsPerWarp; ++rr) {
        const int ry = warp * kStemRowsPerWarp + rr, oy = oy0 + ry;
        if (oy >= Ho) break;
#pragma unroll
        for (int m = 0; m < kStemTW / 16; ++m) {
            // Rows qg and qg + 8 of this MMA tile: output columns ox0 + 16 m + {qg, qg + 8}.
            const int base0 = ((2 * ry) * kStemIW + 2 * (16 * m + qg)) * kStemCin;
            const int base1 = base0 + 2 * 8 * kStemCin;
            float acc[NT][4];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                __nv_bfloat16 e0[4], e1[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __nv_bfloat16 z = __float2bfloat16_rn(0.f);
                    e0[j] = koff[s][j] >= 0 ? xs[base0 + koff[s][j]] : z;
                    e1[j] = koff[s][j] >= 0 ? xs[base1 + koff[s][j]] : z;
                }
                const uint32_t a[4] = {pack_bf16x2(e0[0], e0[1]), pack_bf16x2(e1[0], e1[1]),
                                       pack_bf16x2(e0[2], e0[3]), pack_bf16x2(e1[2], e1[3])};
#pragma unroll
                for (int t = 0; t < NT; ++t) mma_16816(acc[t], a, bf[t][s][0], bf[t][s][1]);
            }
            // Epilogue: round the convolution to bf16, add the bias, GELU, round once more.
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int ox = ox0 + 16 * m + qg + 8 * h;
                if (ox >= Wo) continue;
                YT* yp = y + (((int64_t)b * Ho + oy) * Wo + ox) * COUT + 2 * qt;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float2 r = __bfloat1622float2(__floats2bfloat162_rn(acc[t][2 * h], acc[t][2 * h + 1]));
                    float2 v = make_float2(r.x + bv[t][0], r.y + bv[t][1]);
                    if (GELU) v = gelu2(v);
                    if constexpr (std::is_same<YT, float>::value) {
                        *reinterpret_cast<float2*>(yp + 8 * t) = v;
                    } else {
                        *reinterpret_cast<__nv_bfloat162*>(yp + 8 * t) = __floats2bfloat162_rn(v.x, v.y);
                    }
                }
            }
        }
    }
}

template <int NT, typename YT>
int stem_run(const float* x, const float* w, const float* bias, void* y, int B, int H, int W, int act,
             cudaStream_t st) {
    const int Ho = (H - 1) / 2 + 1, Wo = (W - 1) / 2 + 1;
    const int tiles_w = (Wo + kStemTW - 1) / kStemTW, tiles_h = (Ho + kStemTH - 1) / kStemTH;
    const dim3 grid(tiles_w * tiles_h, B);
    if (act == VH_ACT_GELU)
        stem_conv_kernel<NT, true, YT><<<grid, 32 * kStemWarps, 0, st>>>(x, w, bias, static_cast<YT*>(y), H, W, Ho,
                                                                         Wo, tiles_w);
    else
        stem_conv_kernel<NT, false, YT><<<grid, 32 * kStemWarps, 0, st>>>(x, w, bias, static_cast<YT*>(y), H, W, Ho,
                                                                          Wo, tiles_w);
    return launch_status("stem conv");
}

template <typename YT>
int stem_nt(int cout, const float* x, const float* w, const float* bias, void* y, int B, int H, int W, int act,
            cudaStream_t st) {
    switch (cout) {
        case 16: return stem_run<2, YT>(x, w, bias, y, B, H, W, act, st);
        case 24: return stem_run<3, YT>(x, w, bias, y, B, H, W, act, st);
        case 32: return stem_run<4, YT>(x, w, bias, y, B, H, W, act, st);
        case 48: return stem_run<6, YT>(x, w, bias, y, B, H, W, act, st);
        default: return stem_run<8, YT>(x, w, bias, y, B, H, W, act, st);
    }
}

}  // namespace
}  // namespace vh

using namespace vh;

extern "C" int vh_stem_conv_fwd(const float* x, const float* weight, const float* bias, void* y, int32_t y_dtype,
                                int32_t batch, int32_t height, int32_t width, int32_t out_channels, int32_t act,
                                vh_stream_t stream) {
    clear_error();
    if (!x || !weight || !bias || !y) return fail(VH_E_ARG, "vh_stem_conv_fwd: null pointer argument");
    if (y_dtype != VH_F32 && y_dtype != VH_BF16) return fail(VH_E_DTYPE, "vh_stem_conv_fwd: y must be fp32 or bf16");
    if (act != VH_ACT_NONE && act != VH_ACT_GELU) return fail(VH_E_ARG, "vh_stem_conv_fwd: bad activation %d", act);
    if (batch <= 0 || height <= 0 || width <= 0) return fail(VH_E_SHAPE, "vh_stem_conv_fwd: empty input");
    if (out_channels != 16 && out_channels != 24 && out_channels != 32 && out_channels != 48 && out_channels != 64)
        return fail(VH_E_SHAPE, "vh_stem_conv_fwd: out_channels must be 16, 24, 32, 48 or 64 (got %d)", out_channels);
    if (batch > 65535) return fail(VH_E_RANGE, "vh_stem_conv_fwd: batch must be <= 65535");
    if (!aligned(x, 4) || !aligned(y, 8) || !aligned(weight, 4) || !aligned(bias, 4))
        return fail(VH_E_ALIGN, "vh_stem_conv_fwd: misaligned pointers");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return y_dtype == VH_F32 ? stem_nt<float>(out_channels, x, weight, bias, y, batch, height, width, act, st)
                             : stem_nt<__nv_bfloat16>(out_channels, x, weight, bias, y, batch, height, width, act, st);
}
