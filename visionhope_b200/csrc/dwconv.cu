// Depthwise KxK convolutions of the VisionHOPE block with fused epilogues (sm_100a).
//
// The block (models/block.py) runs four depthwise convolutions per layer, each followed by
// elementwise work that PyTorch issues as separate passes over HBM:
//   cpe             x + (conv3x3(x) + b)                          block.py:100
//                   (optionally of s = x + r: the previous block's pending FFN residual)
//   local features  inner + sigmoid(gate) * (conv7x7(inner) + b)  block.py:57-62
//   output position conv5x5(x_local) + b                          block.py:78
//   FFN             h = gelu(fc1); gelu(h + conv3x3(h) + b)        layers.py (FeedForward)
// One kernel per call does the convolution and its epilogue.  A CTA owns a TH x TC pixel tile
// of 32 channels: it stages the tile plus its halo in shared memory as fp32 (one read of the
// input, the loads of a batch issued together), each thread accumulates R output rows of one
// column for 4 channels with packed two-lane FMAs, holding the column's K weights in
// registers so every staged input vector feeds up to K rows, and the epilogue writes each
// output once.  Eight threads cover a pixel's 32 channels, so the 16-byte shared-memory
// reads of a warp are contiguous and free of bank conflicts.
//
// Arithmetic matches a bf16 convolution under autocast: the convolution reads its input,
// weights and bias rounded to bf16 and accumulates in fp32; residual and gate terms use the
// input as given; the result is rounded once to the output dtype (the input dtype).  GELU is
// the exact (erf) form, with erf from Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7, far below
// the bf16 rounding of every GELU output here).
#include <algorithm>
#include <type_traits>

#include "abi_util.h"
#include "common.cuh"
#include "activations.cuh"
#include "f32x2.cuh"

namespace vh {
namespace {

constexpr int kDwCG = 32;  // channels per CTA (a staged pixel is 32 floats)

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float sigmoid_f(float v) {
    return rcp_approx(1.f + ex2_approx(v * -1.4426950408889634f));
}

// Eight consecutive elements held raw in registers between their load and their use.
template <typename T>
struct Raw8;
template <>
struct Raw8<float> {
    float4 a, b;
    __device__ __forceinline__ void load(const float* p) {
        a = __ldg(reinterpret_cast<const float4*>(p));
        b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void to_float(float (&f)[8]) const {
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ __forceinline__ void store_raw(float* p) const {
        reinterpret_cast<float4*>(p)[0] = a;
        reinterpret_cast<float4*>(p)[1] = b;
    }
};
template <>
struct Raw8<__nv_bfloat16> {
    uint4 u;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { u = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void to_float(float (&f)[8]) const { load8(reinterpret_cast<const __nv_bfloat16*>(&u), f); }
    __device__ __forceinline__ void store_raw(__nv_bfloat16* p) const { *reinterpret_cast<uint4*>(p) = u; }
};

// Four channels as two lane pairs.
__device__ __forceinline__ void lds4(const float* p, float2 (&v)[2]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
}

// MI (several images per CTA): the image is R x TC pixels, and row group g of the CTA owns the
// whole of image RG * blockIdx.z + g, staged as its own (R + K - 1) x (TC + K - 1) halo region.
// Small images then fill a CTA: at 7 x 7 a one-image tile spends most of its time on the
// per-CTA fixed costs (weights, barriers, launch).
template <int K, int TC, int RG, int R, bool MI = false>
struct DwGeom {
    static constexpr int TH = RG * R, P = K / 2, SR = R + K - 1;
    static constexpr int IH = MI ? RG * SR : TH + K - 1, IW = TC + K - 1, NT = 8 * TC * RG;
    static constexpr int XS = IH * IW * kDwCG;  // floats of the staged tile
    static constexpr size_t kSmem = sizeof(float) * ((size_t)XS + K * K * kDwCG + kDwCG);
};

// Epilogue operands of the gated mode staged beside the tile during the load phase, so its
// epilogue reads only shared memory: the exact fp32 input of every output pixel when x is fp32
// (the staged tile holds it rounded to bf16), then the gate of every output pixel.  (The
// residual modes read an fp32 centre from global memory: staging it too costs them more
// occupancy than the loads cost.)
template <int K, int MODE, typename T, int TC, int RG, int R, bool MI = false>
struct DwCenter {
    using G = DwGeom<K, TC, RG, R, MI>;
    static constexpr bool kGate = MODE == VH_DW_GATE || MODE == VH_DW_GATE_POS;
    static constexpr bool kExact = std::is_same<T, float>::value && kGate;
    static constexpr size_t kPix = (size_t)G::TH * TC * kDwCG;  // elements per region
    static constexpr size_t kGateOffset = kExact ? kPix * 4 : 0;  // bytes
    static constexpr size_t kBytes = kGateOffset + (kGate ? kPix * sizeof(T) : 0);
    static constexpr size_t kSmem = G::kSmem + kBytes;
};

template <int K, int MODE, typename T, typename GT, int TC, int RG, int R, bool MI = false>
__global__ void __launch_bounds__(8 * TC * RG, (K == 7 && R >= 7) ? 2 : (K == 7 || MODE == VH_DW_GELU) ? 3 : 4) dwconv_kernel(const T* __restrict__ x, const GT* __restrict__ gate,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ bias, T* __restrict__ y,
                                                                float* __restrict__ sumsq,
                                                                int H, int W, int C, int tiles_w, int B,
                                                                const float* __restrict__ pos_w,
                                                                const float* __restrict__ pos_b,
                                                                T* __restrict__ pos_y) {
    using G = DwGeom<K, TC, RG, R, MI>;
    constexpr int TH = G::TH, P = G::P, IW = G::IW, NT = G::NT, SR = G::SR;
    extern __shared__ __align__(16) float dw_smem[];
    float* xs = dw_smem;                  // [IH][IW][32]
    float* ws = dw_smem + G::XS;          // [K*K][32]
    float* bs = ws + K * K * kDwCG;       // [32]
    using CT = DwCenter<K, MODE, T, TC, RG, R, MI>;
    unsigned char* cbuf = reinterpret_cast<unsigned char*>(bs + kDwCG);  // [TH][TC][32] epilogue operands
    const int tid = threadIdx.x;
    // MI: images b0 .. b0 + RG - 1, one per row group; otherwise one tile of image b0.
    const int b0 = MI ? blockIdx.z * RG : blockIdx.z, c0 = blockIdx.y * kDwCG;
    const int oy0 = MI ? 0 : (blockIdx.x / tiles_w) * TH, ox0 = MI ? 0 : (blockIdx.x % tiles_w) * TC;
    const int64_t plane = (int64_t)H * W * C;

    for (int i = tid; i < K * K * kDwCG; i += NT) {
        const int tap = i / kDwCG, cc = i % kDwCG, c = c0 + cc;
        ws[i] = c < C ? round_bf16(w[(int64_t)c * K * K + tap]) : 0.f;
    }
    if (tid < kDwCG) bs[tid] = c0 + tid < C ? round_bf16(bias[c0 + tid]) : 0.f;
    // Input tile with halo, in 8-channel vectors; zero outside the image (the convolution's
    // zero padding).  The loads of a batch are all issued before any of them is converted.
    // Loads per batch: the whole tile at once for the GELU and bias modes (one round trip to
    // HBM); four for the others, whose extra operands would otherwise spill or cost occupancy.
    constexpr int NV = G::IH * IW * 4, IT = (NV + NT - 1) / NT;
    constexpr int BATCH = (MODE == VH_DW_GELU || MODE == VH_DW_BIAS) ? (IT < 8 ? IT : 8) : 4;
#pragma unroll
    for (int i0 = 0; i0 < IT; i0 += BATCH) {
        Raw8<T> raw[BATCH];
        Raw8<GT> rawa[MODE == VH_DW_RESID_ADD ? BATCH : 1];
        Raw8<T> rawg[CT::kGate ? BATCH : 1];
        bool live[BATCH], centre[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
            const int i = (i0 + u) * NT + tid;
            const int v = i & 3, pix = i >> 2;
            const int py = pix / IW, px = pix % IW;
            // MI: staged row py is row ly of the halo region of image b0 + py / SR.
            const int ly = MI ? py % SR : py, bi = MI ? b0 + py / SR : b0;
            const int gy = oy0 + ly - P, gx = ox0 + px - P, c = c0 + 8 * v;
            live[u] = i0 + u < IT && i < NV && gy >= 0 && gy < H && gx >= 0 && gx < W && c < C && bi < B;
            centre[u] = live[u] && ly >= P && ly < P + (MI ? R : TH) && px >= P && px < P + TC;
            const int64_t img = (int64_t)bi * plane;
            if (live[u]) {
                raw[u].load(x + img + ((int64_t)gy * W + gx) * C + c);
                if (MODE == VH_DW_RESID_ADD) rawa[MODE == VH_DW_RESID_ADD ? u : 0].load(gate + img + ((int64_t)gy * W + gx) * C + c);
            }
            if (CT::kGate && centre[u]) rawg[CT::kGate ? u : 0].load(reinterpret_cast<const T*>(gate) + img + ((int64_t)gy * W + gx) * C + c);
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
            const int i = (i0 + u) * NT + tid;
            if (i0 + u >= IT || i >= NV) continue;
            float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (live[u]) {
                raw[u].to_float(f);
                if (MODE == VH_DW_RESID_ADD) {  // the pending residual: s = x + addend
                    float a8[8];
                    rawa[MODE == VH_DW_RESID_ADD ? u : 0].to_float(a8);
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] += a8[e];
                    if (std::is_same<T, __nv_bfloat16>::value) {  // s is stored in x's dtype
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            const float2 r2 = __bfloat1622float2(__floats2bfloat162_rn(f[e], f[e + 1]));
                            f[e] = r2.x;
                            f[e + 1] = r2.y;
                        }
                    }
                }
                if (MODE == VH_DW_GELU) {
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const float2 g = gelu2(make_float2(f[e], f[e + 1]));
                        f[e] = g.x;
                        f[e + 1] = g.y;
                    }
                }
                const int pix = i >> 2, py = pix / IW;
                // output pixel row within the CTA's [TH][TC] operands (MI: image row group first)
                const int orow = MI ? (py / SR) * R + py % SR - P : py - P;
                const int cidx = (orow * TC + (pix % IW - P)) * kDwCG + 8 * (i & 3);
                if (CT::kExact && centre[u]) {  // the exact input of this output pixel
                    float* d = reinterpret_cast<float*>(cbuf) + cidx;
                    reinterpret_cast<float4*>(d)[0] = make_float4(f[0], f[1], f[2], f[3]);
                    reinterpret_cast<float4*>(d)[1] = make_float4(f[4], f[5], f[6], f[7]);
                }
                if (CT::kGate && centre[u])
                    rawg[CT::kGate ? u : 0].store_raw(reinterpret_cast<T*>(cbuf + CT::kGateOffset) + cidx);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {  // packed round to bf16 and back
                    const float2 r = __bfloat1622float2(__floats2bfloat162_rn(f[e], f[e + 1]));
                    f[e] = r.x;
                    f[e + 1] = r.y;
                }
            }
            float* d = xs + (i >> 2) * kDwCG + 8 * (i & 3);
            reinterpret_cast<float4*>(d)[0] = make_float4(f[0], f[1], f[2], f[3]);
            reinterpret_cast<float4*>(d)[1] = make_float4(f[4], f[5], f[6], f[7]);
        }
    }
    __syncthreads();

    const int q = tid & 7, col = (tid >> 3) % TC, rg = (tid >> 3) / TC, r0 = rg * R;
    const int c = c0 + 4 * q, ox = ox0 + col;
    const int b = MI ? b0 + rg : b0;
    const int64_t img = (int64_t)b * plane;
    const bool out_ok = c < C && ox < W && b < B;
    float2 acc[R][2];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = make_float2(0.f, 0.f);
    // Per-thread bases; every shared-memory address below is one of these plus a constant.
    const float* xt = xs + ((MI ? rg * SR : r0) * IW + col) * kDwCG + 4 * q;
    const float* wt = ws + 4 * q;
#pragma unroll
    for (int kx = 0; kx < K; ++kx) {
        float2 wk[K][2];
#pragma unroll
        for (int ky = 0; ky < K; ++ky) lds4(wt + (ky * K + kx) * kDwCG, wk[ky]);
#pragma unroll
        for (int iy = 0; iy < R + K - 1; ++iy) {
            float2 in[2];
            lds4(xt + (iy * IW + kx) * kDwCG, in);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int ky = iy - r;
                if (ky >= 0 && ky < K) {
                    acc[r][0] = ffma2(wk[ky][0], in[0], acc[r][0]);
                    acc[r][1] = ffma2(wk[ky][1], in[1], acc[r][1]);
                }
            }
        }
    }

    // GELU mode with `sumsq`: this thread's sums of y^2 (as stored) over its rows, 4 channels.
    float2 ss[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    // GATE_POS: this thread's outputs as stored (bf16-rounded), the position conv's input.
    constexpr int KR = MODE == VH_DW_GATE_POS ? R : 1;
    float2 keep[KR][2];
#pragma unroll
    for (int r = 0; r < KR; ++r) keep[r][0] = keep[r][1] = make_float2(0.f, 0.f);
    float2 bv[2];
    lds4(bs + 4 * q, bv);
    const int64_t off0 = img + ((int64_t)(oy0 + (MI ? 0 : r0)) * W + ox) * C + c, row = (int64_t)W * C;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int oy = oy0 + (MI ? 0 : r0) + r;
        if (!out_ok || oy >= H) break;
        const int64_t off = off0 + r * row;
        float2 o[2] = {fadd2(acc[r][0], bv[0]), fadd2(acc[r][1], bv[1])};
        if (MODE == VH_DW_RESID || MODE == VH_DW_RESID_ADD || CT::kGate) {
            // The centre value itself: from the staged tile when the input is bf16 (staged
            // exactly), else from the exact copy staged for the gated epilogue, or from global
            // memory.
            float2 xc[2];
            const int cidx = ((r0 + r) * TC + col) * kDwCG + 4 * q;
            if (std::is_same<T, __nv_bfloat16>::value) {
                lds4(xt + ((r + P) * IW + P) * kDwCG, xc);
            } else if (CT::kExact) {
                lds4(reinterpret_cast<const float*>(cbuf) + cidx, xc);
            } else {
                float4 t4 = load4(x + off);
                if (MODE == VH_DW_RESID_ADD) {
                    const float4 a4 = load4(gate + off);
                    t4 = make_float4(t4.x + a4.x, t4.y + a4.y, t4.z + a4.z, t4.w + a4.w);
                }
                xc[0] = make_float2(t4.x, t4.y);
                xc[1] = make_float2(t4.z, t4.w);
            }
            if (!CT::kGate) {
                o[0] = fadd2(xc[0], o[0]);
                o[1] = fadd2(xc[1], o[1]);
            } else {
                const float4 g = load4(reinterpret_cast<const T*>(cbuf + CT::kGateOffset) + cidx);
                o[0] = ffma2(make_float2(sigmoid_f(g.x), sigmoid_f(g.y)), o[0], xc[0]);
                o[1] = ffma2(make_float2(sigmoid_f(g.z), sigmoid_f(g.w)), o[1], xc[1]);
            }
        } else if (MODE == VH_DW_GELU) {
            float2 h[2];  // gelu(x) at the centre, as staged
            lds4(xt + ((r + P) * IW + P) * kDwCG, h);
            o[0] = gelu2(fadd2(h[0], o[0]));
            o[1] = gelu2(fadd2(h[1], o[1]));
            if constexpr (std::is_same<T, __nv_bfloat16>::value) {
                // Round once: the stored pair is also what the GRN sums see.
                const __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0].x, o[0].y);
                const __nv_bfloat162 p1 = __floats2bfloat162_rn(o[1].x, o[1].y);
                *reinterpret_cast<uint2*>(y + off) = make_uint2(*reinterpret_cast<const uint32_t*>(&p0),
                                                                *reinterpret_cast<const uint32_t*>(&p1));
                if (sumsq) {
                    const float2 s0 = __bfloat1622float2(p0), s1 = __bfloat1622float2(p1);
                    ss[0] = ffma2(s0, s0, ss[0]);
                    ss[1] = ffma2(s1, s1, ss[1]);
                }
                continue;
            }
            ss[0] = ffma2(o[0], o[0], ss[0]);
            ss[1] = ffma2(o[1], o[1], ss[1]);
        }
        if constexpr (MODE == VH_DW_GATE_POS) {
            keep[MODE == VH_DW_GATE_POS ? r : 0][0] = make_float2(round_bf16(o[0].x), round_bf16(o[0].y));
            keep[MODE == VH_DW_GATE_POS ? r : 0][1] = make_float2(round_bf16(o[1].x), round_bf16(o[1].y));
        }
        store4(y + off, make_float4(o[0].x, o[0].y, o[1].x, o[1].y));
    }
    if constexpr (MODE == VH_DW_GATE_POS) {
        // The output position term: a K2 x K2 convolution of y (as stored) with its own weights
        // and bias, from a copy of this CTA's outputs in shared memory.  The CTA holds whole
        // images, so the copy's zero border is the convolution's zero padding, and the sums run
        // in the order of the VH_DW_BIAS mode: bit-identical to that mode applied to y.
        constexpr int K2 = 5, P2 = K2 / 2, SR2 = R + K2 - 1, IW2 = TC + K2 - 1;
        constexpr int IH2 = MI ? RG * SR2 : TH + K2 - 1, OH = MI ? R : TH;
        static_assert(IH2 * IW2 <= G::IH * IW, "the position input fits where the tile was staged");
        static_assert(K2 <= K, "the position weights fit where the first weights were staged");
        __syncthreads();  // every read of the staged tile, weights and bias is done
        float* ps = xs;   // [IH2][IW2][32]
        for (int i = tid; i < IH2 * IW2 * 8; i += NT) {
            const int pix = i >> 3, py = pix / IW2, px = pix % IW2, ly = MI ? py % SR2 : py;
            if (ly < P2 || ly >= P2 + OH || px < P2 || px >= P2 + TC)
                *reinterpret_cast<float4*>(ps + pix * kDwCG + 4 * (i & 7)) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int prow = MI ? rg * SR2 : r0;  // this thread's first row in the copy, less P2
#pragma unroll
        for (int r = 0; r < R; ++r)
            *reinterpret_cast<float4*>(ps + ((prow + P2 + r) * IW2 + col + P2) * kDwCG + 4 * q) =
                make_float4(keep[r][0].x, keep[r][0].y, keep[r][1].x, keep[r][1].y);
        for (int i = tid; i < K2 * K2 * kDwCG; i += NT) {
            const int tap = i / kDwCG, cc = i % kDwCG, ch = c0 + cc;
            ws[i] = ch < C ? round_bf16(pos_w[(int64_t)ch * K2 * K2 + tap]) : 0.f;
        }
        if (tid < kDwCG) bs[tid] = c0 + tid < C ? round_bf16(pos_b[c0 + tid]) : 0.f;
        __syncthreads();
        float2 acc2[R][2];
#pragma unroll
        for (int r = 0; r < R; ++r) acc2[r][0] = acc2[r][1] = make_float2(0.f, 0.f);
        const float* pt = ps + (prow * IW2 + col) * kDwCG + 4 * q;
#pragma unroll
        for (int kx = 0; kx < K2; ++kx) {
            float2 wk[K2][2];
#pragma unroll
            for (int ky = 0; ky < K2; ++ky) lds4(wt + (ky * K2 + kx) * kDwCG, wk[ky]);
#pragma unroll
            for (int iy = 0; iy < R + K2 - 1; ++iy) {
                float2 in[2];
                lds4(pt + (iy * IW2 + kx) * kDwCG, in);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int ky = iy - r;
                    if (ky >= 0 && ky < K2) {
                        acc2[r][0] = ffma2(wk[ky][0], in[0], acc2[r][0]);
                        acc2[r][1] = ffma2(wk[ky][1], in[1], acc2[r][1]);
                    }
                }
            }
        }
        float2 bv2[2];
        lds4(bs + 4 * q, bv2);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int oy = oy0 + (MI ? 0 : r0) + r;
            if (!out_ok || oy >= H) break;
            const float2 o0 = fadd2(acc2[r][0], bv2[0]), o1 = fadd2(acc2[r][1], bv2[1]);
            store4(pos_y + off0 + r * row, make_float4(o0.x, o0.y, o1.x, o1.y));
        }
    }
    if (MI && MODE == VH_DW_GELU && sumsq) {
        // Per-image channel sums in a fixed order (the columns of the image's row group; a row
        // group need not start on a warp boundary, so the sums go through shared memory).
        __syncthreads();
        *reinterpret_cast<float4*>(xs + 4 * tid) = make_float4(ss[0].x, ss[0].y, ss[1].x, ss[1].y);
        __syncthreads();
        if (tid < RG * kDwCG) {
            const int g = tid / kDwCG, ch = tid % kDwCG, bi = b0 + g;
            float t = 0.f;
#pragma unroll
            for (int cc = 0; cc < TC; ++cc) t += xs[4 * ((g * TC + cc) * 8 + ch / 4) + ch % 4];
            if (bi < B && c0 + ch < C) sumsq[(int64_t)bi * C + c0 + ch] = t;
        }
    } else if (MODE == VH_DW_GELU && sumsq) {
        // Per-tile channel sums in a fixed order: the four lanes of a warp that share channels
        // (lane bits 3-4), then the warps in index order; the staged tile is free by now.
#pragma unroll
        for (int m = 8; m <= 16; m <<= 1) {
            ss[0].x += __shfl_xor_sync(0xffffffffu, ss[0].x, m);
            ss[0].y += __shfl_xor_sync(0xffffffffu, ss[0].y, m);
            ss[1].x += __shfl_xor_sync(0xffffffffu, ss[1].x, m);
            ss[1].y += __shfl_xor_sync(0xffffffffu, ss[1].y, m);
        }
        __syncthreads();
        const int lane = tid & 31, warp = tid >> 5;
        if (lane < 8) *reinterpret_cast<float4*>(xs + warp * kDwCG + 4 * lane) = make_float4(ss[0].x, ss[0].y, ss[1].x, ss[1].y);
        __syncthreads();
        if (tid < kDwCG && c0 + tid < C) {
            float t = 0.f;
#pragma unroll
            for (int w8 = 0; w8 < NT / 32; ++w8) t += xs[w8 * kDwCG + tid];
            sumsq[((int64_t)b * gridDim.x + blockIdx.x) * C + c0 + tid] = t;
        }
    }
}

template <int K, int MODE, typename T, typename GT, int TC, int RG, int R, bool MI = false>
int dw_launch(const vh_dwconv_args& a, cudaStream_t st) {
    using G = DwGeom<K, TC, RG, R, MI>;
    const int tiles_w = MI ? 1 : (a.width + TC - 1) / TC, tiles_h = MI ? 1 : (a.height + G::TH - 1) / G::TH;
    const dim3 grid(tiles_w * tiles_h, (a.channels + kDwCG - 1) / kDwCG, MI ? (a.batch + RG - 1) / RG : a.batch);
    const void* fn = reinterpret_cast<const void*>(&dwconv_kernel<K, MODE, T, GT, TC, RG, R, MI>);
    constexpr size_t smem = DwCenter<K, MODE, T, TC, RG, R, MI>::kSmem;
    if (!ensure_smem_attr(fn, smem))
        return fail(VH_E_DEVICE, "depthwise conv: cannot reserve %zu bytes of shared memory", smem);
    dwconv_kernel<K, MODE, T, GT, TC, RG, R, MI><<<grid, G::NT, smem, st>>>(
        static_cast<const T*>(a.x), static_cast<const GT*>(a.gate), a.weight, a.bias, static_cast<T*>(a.y),
        MODE == VH_DW_GELU ? a.sumsq : nullptr, a.height, a.width, a.channels, tiles_w, a.batch, a.pos_weight,
        a.pos_bias, static_cast<T*>(a.pos_y));
    return launch_status("depthwise conv");
}

// Tile: the shape among 14 x 14 (224 threads, 7 rows each; divides every VisionHOPE stage
// size from 14 up), 16 x 16 (256 threads, 8 rows each) and 8 x 8 (256 threads, 2 rows each)
// that covers the image with the least padding, in that order of preference.
inline int dw_tile_side(int H, int W) {
    auto area = [&](int t) { return (int64_t)((H + t - 1) / t) * t * (int64_t)((W + t - 1) / t) * t; };
    const int64_t a14 = area(14), a16 = area(16), a8 = area(8);
    if (a14 <= a16 && a14 <= a8) return 14;
    return a16 <= a8 ? 16 : 8;
}

// Images of 7 x 7 pixels (the last stage at 224 x 224): four whole images per CTA.
constexpr int kDwMiImages = 4;

template <int K, int MODE, typename T, typename GT>
int dw_tile(const vh_dwconv_args& a, cudaStream_t st) {
    if (a.height == 7 && a.width == 7) return dw_launch<K, MODE, T, GT, 7, kDwMiImages, 7, true>(a, st);
    switch (dw_tile_side(a.height, a.width)) {
        case 14: return dw_launch<K, MODE, T, GT, 14, 2, 7>(a, st);
        case 16: return dw_launch<K, MODE, T, GT, 16, 2, 8>(a, st);
        default: return dw_launch<K, MODE, T, GT, 8, 4, 2>(a, st);
    }
}

template <int MODE, typename T, typename GT = T>
int dw_k(const vh_dwconv_args& a, cudaStream_t st) {
    switch (a.ksize) {
        case 3: return dw_tile<3, MODE, T, GT>(a, st);
        case 5: return dw_tile<5, MODE, T, GT>(a, st);
        default: return dw_tile<7, MODE, T, GT>(a, st);
    }
}

// The gated local features and the output position term in one pass: bf16, 7x7 then 5x5,
// whole images per CTA (the 14 x 14 tile of a 14 x 14 image, or four 7 x 7 images).
template <typename T>
int dw_gate_pos(const vh_dwconv_args& a, cudaStream_t st) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        if (a.height == 7 && a.width == 7) return dw_launch<7, VH_DW_GATE_POS, T, T, 7, kDwMiImages, 7, true>(a, st);
        return dw_launch<7, VH_DW_GATE_POS, T, T, 14, 2, 7>(a, st);
    }
    return fail(VH_E_DTYPE, "vh_dwconv_fwd: VH_DW_GATE_POS needs bf16");
}

template <typename T>
int dw_mode(const vh_dwconv_args& a, cudaStream_t st) {
    switch (a.mode) {
        case VH_DW_GATE_POS: return dw_gate_pos<T>(a, st);
        case VH_DW_BIAS: return dw_k<VH_DW_BIAS, T>(a, st);
        case VH_DW_RESID: return dw_k<VH_DW_RESID, T>(a, st);
        case VH_DW_GATE: return dw_k<VH_DW_GATE, T>(a, st);
        case VH_DW_RESID_ADD:
            return a.gate_dtype == VH_F32 ? dw_k<VH_DW_RESID_ADD, T, float>(a, st)
                                          : dw_k<VH_DW_RESID_ADD, T, __nv_bfloat16>(a, st);
        default: return dw_k<VH_DW_GELU, T>(a, st);
    }
}

// Shared-memory limit of one instantiation (the carveout stays the driver's choice: forcing
// the largest shared-memory share slows these kernels, whose halo loads hit in L1).
void dw_attr_one(const void* fn, size_t smem) { ensure_smem_attr(fn, smem); }

template <int K, int MODE, typename T, typename GT>
void dw_attr_k() {
    dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<K, MODE, T, GT, 14, 2, 7>), DwCenter<K, MODE, T, 14, 2, 7>::kSmem);
    dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<K, MODE, T, GT, 16, 2, 8>), DwCenter<K, MODE, T, 16, 2, 8>::kSmem);
    dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<K, MODE, T, GT, 8, 4, 2>), DwCenter<K, MODE, T, 8, 4, 2>::kSmem);
    dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<K, MODE, T, GT, 7, kDwMiImages, 7, true>),
                DwCenter<K, MODE, T, 7, kDwMiImages, 7, true>::kSmem);
}

template <int MODE, typename T, typename GT = T>
void dw_attr_mode() {
    dw_attr_k<3, MODE, T, GT>();
    dw_attr_k<5, MODE, T, GT>();
    dw_attr_k<7, MODE, T, GT>();
}

template <typename T>
void dw_attr_t() {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<7, VH_DW_GATE_POS, T, T, 14, 2, 7>),
                    DwCenter<7, VH_DW_GATE_POS, T, 14, 2, 7>::kSmem);
        dw_attr_one(reinterpret_cast<const void*>(&dwconv_kernel<7, VH_DW_GATE_POS, T, T, 7, kDwMiImages, 7, true>),
                    DwCenter<7, VH_DW_GATE_POS, T, 7, kDwMiImages, 7, true>::kSmem);
    }
    dw_attr_mode<VH_DW_BIAS, T>();
    dw_attr_mode<VH_DW_RESID, T>();
    dw_attr_mode<VH_DW_GATE, T>();
    dw_attr_mode<VH_DW_GELU, T>();
    dw_attr_mode<VH_DW_RESID_ADD, T, float>();
    dw_attr_mode<VH_DW_RESID_ADD, T, __nv_bfloat16>();
}

}  // namespace

// Shared-memory limits of every depthwise kernel on the current device (from vh_init, so a
// first call inside a CUDA-graph capture sets no attribute).
int init_dw_kernels() {
    dw_attr_t<float>();
    dw_attr_t<__nv_bfloat16>();
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(VH_E_DEVICE, "vh_init: %s", cudaGetErrorString(e));
    return 0;
}

}  // namespace vh

using namespace vh;

extern "C" int vh_dwconv_tiles(int32_t height, int32_t width) {
    if (height <= 0 || width <= 0) return 0;
    if (height == 7 && width == 7) return 1;  // whole images per CTA
    const int t = dw_tile_side(height, width);
    return ((height + t - 1) / t) * ((width + t - 1) / t);
}

extern "C" int vh_dwconv_fwd(const vh_dwconv_args* a, vh_stream_t stream) {
    clear_error();
    if (!a) return fail(VH_E_ARG, "vh_dwconv_fwd: null args");
    if (!a->x || !a->weight || !a->bias || !a->y ||
        ((a->mode == VH_DW_GATE || a->mode == VH_DW_GATE_POS || a->mode == VH_DW_RESID_ADD) && !a->gate))
        return fail(VH_E_ARG, "vh_dwconv_fwd: null pointer argument");
    if (a->mode < VH_DW_BIAS || a->mode > VH_DW_GATE_POS) return fail(VH_E_ARG, "vh_dwconv_fwd: bad mode %d", a->mode);
    if (a->mode == VH_DW_GATE_POS) {
        if (!a->pos_weight || !a->pos_bias || !a->pos_y)
            return fail(VH_E_ARG, "vh_dwconv_fwd: VH_DW_GATE_POS needs pos_weight, pos_bias and pos_y");
        if (a->dtype != VH_BF16) return fail(VH_E_DTYPE, "vh_dwconv_fwd: VH_DW_GATE_POS needs bf16");
        if (a->ksize != 7 || a->pos_ksize != 5)
            return fail(VH_E_SHAPE, "vh_dwconv_fwd: VH_DW_GATE_POS takes ksize 7 and pos_ksize 5");
        if (!((a->height == 14 && a->width == 14) || (a->height == 7 && a->width == 7)))
            return fail(VH_E_SHAPE, "vh_dwconv_fwd: VH_DW_GATE_POS needs 14 x 14 or 7 x 7 images (got %d x %d)",
                        a->height, a->width);
        if (!aligned(a->pos_y, 16)) return fail(VH_E_ALIGN, "vh_dwconv_fwd: pos_y must be 16-byte aligned");
        if (a->pos_y == a->x || a->pos_y == a->gate || a->pos_y == a->y)
            return fail(VH_E_ARG, "vh_dwconv_fwd: pos_y must not alias x, gate or y");
    }
    if (a->mode == VH_DW_RESID_ADD && a->gate_dtype != VH_F32 && a->gate_dtype != VH_BF16)
        return fail(VH_E_DTYPE, "vh_dwconv_fwd: the addend must be fp32 or bf16");
    if (a->mode == VH_DW_RESID_ADD && a->dtype == VH_BF16 && a->gate_dtype == VH_F32)
        return fail(VH_E_DTYPE, "vh_dwconv_fwd: an fp32 addend needs fp32 x");
    if (a->ksize != 3 && a->ksize != 5 && a->ksize != 7)
        return fail(VH_E_SHAPE, "vh_dwconv_fwd: kernel size must be 3, 5 or 7 (got %d)", a->ksize);
    if (a->dtype != VH_F32 && a->dtype != VH_BF16)
        return fail(VH_E_DTYPE, "vh_dwconv_fwd: dtype must be fp32 or bf16");
    if (a->batch <= 0 || a->height <= 0 || a->width <= 0 || a->channels <= 0)
        return fail(VH_E_SHAPE, "vh_dwconv_fwd: sizes must be positive");
    if (a->channels % 8) return fail(VH_E_SHAPE, "vh_dwconv_fwd: channels must be a multiple of 8");
    if (a->batch > 65535 || (int64_t)a->height * a->width > ((int64_t)1 << 30))
        return fail(VH_E_RANGE, "vh_dwconv_fwd: sizes exceed the supported range");
    if (!aligned(a->x, 16) || !aligned(a->y, 16) || (a->gate && !aligned(a->gate, 16)))
        return fail(VH_E_ALIGN, "vh_dwconv_fwd: x, gate and y must be 16-byte aligned");
    if (a->sumsq && a->mode != VH_DW_GELU)
        return fail(VH_E_ARG, "vh_dwconv_fwd: sumsq goes with the GELU epilogue");
    if (a->sumsq && !aligned(a->sumsq, 4)) return fail(VH_E_ALIGN, "vh_dwconv_fwd: misaligned sumsq");
    if (a->x == a->y || (a->gate && a->gate == a->y))
        return fail(VH_E_ARG, "vh_dwconv_fwd: y must not alias the inputs");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return a->dtype == VH_F32 ? dw_mode<float>(*a, st) : dw_mode<__nv_bfloat16>(*a, st);
}
