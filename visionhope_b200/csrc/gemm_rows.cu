// Skinny row GEMM for the block's 1x1 projections: y[M, N] = x[M, K] W[N, K]^T + b, bf16 in and
// out, fp32 accumulation (the arithmetic of F.linear under bf16 autocast: fp32 sums, the bf16
// bias added in fp32, one rounding).
//
// The VisionHOPE block's projections have K, N <= 256 and millions of rows, so they are
// bounded by HBM, not by the tensor cores: the kernel is shaped to stream x once at full
// bandwidth.  The weights (at most 64 KB) sit in shared memory for the whole CTA; each warp
// walks 16-row tiles of x and feeds `mma.sync.m16n8k16` straight from 16-byte global loads:
//
//   Within each 32-channel slice, lane (g, q) of the MMA fragment holds rows g and g + 8 of the
//   tile and the logical K indices {2q, 2q+1, 2q+8, 2q+9} of two 16-wide K steps.  The kernel
//   assigns those eight logical indices to the eight consecutive physical channels 8q .. 8q+7,
//   for x and for W alike.  The dot product is a sum over all channels, so any bijection used
//   for both operands gives the same result, and then each lane's A fragment for a slice is
//   one 16-byte load per row, and its B fragment one 16-byte shared-memory read of a W row.
//
// With a LayerNorm prologue (the block's norm1 -> proj_in, models/block.py:104 with
// layers.py:9-35) x is the fp32 residual stream and each row is normalized on its way into the
// A fragments: a row's K channels sit in the four lanes of one MMA row group, so its mean and
// variance take two quad shuffles.  Each normalized value is rounded to bf16 as the LayerNorm
// kernel would store it for the projection, so the GEMM sees the same operand; the normalized
// activations never go to HBM.
#include <atomic>
#include <algorithm>

#include "abi_util.h"
#include "common.cuh"
#include "srnl_scan.cuh"

namespace vh {
namespace {

constexpr int kRgWarps = 8;
constexpr int kRgThreads = 32 * kRgWarps;
constexpr int kRgNGroup = 64;  // output columns per accumulation pass (8 n-tiles)

template <int K, int N>
struct RgGeom {
    // Padded W row (bf16): a row stride of 64 bytes modulo 128 puts the 16-byte reads of the
    // 8 lanes of one shared-memory phase (2 rows x 4 slices) in distinct banks.
    static constexpr int KP = K % 64 == 0 ? K + 32 : K;
    static constexpr size_t kSmem = (size_t)N * KP * 2 + (size_t)N * 4;
    static constexpr size_t kSmemLn = kSmem + (size_t)K * 8;  // + LayerNorm weight and bias (fp32)
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}

// x: bf16 rows, or with LN fp32 rows normalized by (lnw, lnb, eps) first.
template <int K, int N, bool LN>
__global__ void __launch_bounds__(kRgThreads, 2) rows_gemm_kernel(const void* __restrict__ xv,
                                                                  const float* __restrict__ lnw,
                                                                  const float* __restrict__ lnb, float eps,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  const float* __restrict__ bias,
                                                                  __nv_bfloat16* __restrict__ y, int64_t M) {
    using G = RgGeom<K, N>;
    constexpr int KC = K / 32;                       // 32-channel slices
    constexpr int NG = N < kRgNGroup ? N : kRgNGroup;
    constexpr int NT = NG / 8;                       // n-tiles per pass
    extern __shared__ __align__(16) unsigned char rg_smem[];
    __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(rg_smem);          // [N][KP]
    float* bs = reinterpret_cast<float*>(rg_smem + (size_t)N * G::KP * 2);  // [N]
    float* lws = bs + N;                                                    // [K] (LN)
    float* lbs = lws + K;                                                   // [K] (LN)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3;

    // W goes to shared memory as asynchronous 16-byte copies, all in flight at once; the CTA
    // waits for them only after its warps have issued the loads of their first x tile.
    for (int i = tid; i < N * K / 8; i += kRgThreads) {
        const int n = i / (K / 8), k8 = i % (K / 8);
        cp_async<16>(ws + n * G::KP + 8 * k8, w + (int64_t)n * K + 8 * k8);
    }
    cp_async_commit();
    for (int n = tid; n < N; n += kRgThreads) bs[n] = bias ? bias[n] : 0.f;
    if constexpr (LN) {
        for (int k = tid; k < K; k += kRgThreads) {
            lws[k] = lnw[k];
            lbs[k] = lnb[k];
        }
    }
    // Every warp runs the tile loop at least once (an iteration past the last tile loads and
    // stores nothing), so every thread reaches this barrier exactly once.
    bool first = true;
    auto weights_ready = [&]() {
        if (first) {
            cp_async_wait<0>();
            __syncthreads();
            first = false;
        }
    };

    // A warp takes MT 16-row tiles at a time (every B fragment read from shared memory then
    // feeds 2 MT MMAs).  One tile measured fastest at the shapes this kernel serves: more tiles
    // per warp cost registers and CTAs that the loads in flight do not recover.
    constexpr int MT = 1;
    const int64_t groups = (M + 16 * MT - 1) / (16 * MT);
    for (int64_t grp = (int64_t)blockIdx.x * kRgWarps + warp; first || grp < groups;
         grp += (int64_t)gridDim.x * kRgWarps) {
        uint4 a0[MT][KC], a1[MT][KC];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const int64_t r0 = (grp * MT + m) * 16 + g, r1 = r0 + 8;
            if constexpr (!LN) {
                const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(xv);
#pragma unroll
                for (int c = 0; c < KC; ++c) {
                    a0[m][c] = r0 < M ? __ldcs(reinterpret_cast<const uint4*>(x + r0 * K + 32 * c + 8 * q)) : make_uint4(0, 0, 0, 0);
                    a1[m][c] = r1 < M ? __ldcs(reinterpret_cast<const uint4*>(x + r1 * K + 32 * c + 8 * q)) : make_uint4(0, 0, 0, 0);
                }
                weights_ready();
            } else {
                // This lane's 8 channels of each slice for rows r0 and r1, then each row's
                // statistics over its four lanes: mean, then the centred sum of squares, and
                // rstd = 1 / sqrt(var + eps) (biased variance, as the LayerNorm kernel).
                const float* x = static_cast<const float*>(xv);
                float v[2][KC][8];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int64_t r = h ? r1 : r0;
#pragma unroll
                    for (int c = 0; c < KC; ++c) {
                        float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
                        if (r < M) {
                            const float4* src = reinterpret_cast<const float4*>(x + r * K + 32 * c + 8 * q);
                            lo = __ldcs(src);
                            hi = __ldcs(src + 1);
                        }
                        v[h][c][0] = lo.x; v[h][c][1] = lo.y; v[h][c][2] = lo.z; v[h][c][3] = lo.w;
                        v[h][c][4] = hi.x; v[h][c][5] = hi.y; v[h][c][6] = hi.z; v[h][c][7] = hi.w;
                    }
                }
                weights_ready();  // also orders the LayerNorm parameters written above
                float mean[2], rstd[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float sum = 0.f;
#pragma unroll
                    for (int c = 0; c < KC; ++c)
                        sum += ((v[h][c][0] + v[h][c][1]) + (v[h][c][2] + v[h][c][3])) +
                               ((v[h][c][4] + v[h][c][5]) + (v[h][c][6] + v[h][c][7]));
                    mean[h] = quad_sum(sum) / (float)K;
                    float sq = 0.f;
#pragma unroll
                    for (int c = 0; c < KC; ++c)
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float d = v[h][c][e] - mean[h];
                            sq = fmaf(d, d, sq);
                        }
                    rstd[h] = 1.f / sqrtf(quad_sum(sq) * (1.f / (float)K) + eps);
                }
#pragma unroll
                for (int c = 0; c < KC; ++c) {
                    const int k0 = 32 * c + 8 * q;
                    const float4 wl = *reinterpret_cast<const float4*>(lws + k0), wh = *reinterpret_cast<const float4*>(lws + k0 + 4);
                    const float4 bl = *reinterpret_cast<const float4*>(lbs + k0), bh = *reinterpret_cast<const float4*>(lbs + k0 + 4);
                    const float lw[8] = {wl.x, wl.y, wl.z, wl.w, wh.x, wh.y, wh.z, wh.w};
                    const float lb[8] = {bl.x, bl.y, bl.z, bl.w, bh.x, bh.y, bh.z, bh.w};
                    uint32_t pk[2][4];
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int e = 0; e < 8; e += 2)
                            pk[h][e / 2] = pack_bf16x2((v[h][c][e] - mean[h]) * rstd[h] * lw[e] + lb[e],
                                                       (v[h][c][e + 1] - mean[h]) * rstd[h] * lw[e + 1] + lb[e + 1]);
                    a0[m][c] = make_uint4(pk[0][0], pk[0][1], pk[0][2], pk[0][3]);
                    a1[m][c] = make_uint4(pk[1][0], pk[1][1], pk[1][2], pk[1][3]);
                }
            }
        }
#pragma unroll
        for (int n0 = 0; n0 < N; n0 += NG) {
            float acc[MT][NT][4];
#pragma unroll
            for (int m = 0; m < MT; ++m)
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[m][t][0] = acc[m][t][1] = acc[m][t][2] = acc[m][t][3] = 0.f;
#pragma unroll
            for (int c = 0; c < KC; ++c) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint4 b = *reinterpret_cast<const uint4*>(ws + (n0 + 8 * t + g) * G::KP + 32 * c + 8 * q);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint32_t A0[4] = {a0[m][c].x, a1[m][c].x, a0[m][c].y, a1[m][c].y};
                        const uint32_t A1[4] = {a0[m][c].z, a1[m][c].z, a0[m][c].w, a1[m][c].w};
                        mma_16816(acc[m][t], A0, b.x, b.y);
                        mma_16816(acc[m][t], A1, b.z, b.w);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int64_t r0 = (grp * MT + m) * 16 + g, r1 = r0 + 8;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const int col = n0 + 8 * t + 2 * q;
                    const float b0 = bs[col], b1 = bs[col + 1];
                    if (r0 < M)
                        *reinterpret_cast<__nv_bfloat162*>(y + r0 * N + col) =
                            __floats2bfloat162_rn(acc[m][t][0] + b0, acc[m][t][1] + b1);
                    if (r1 < M)
                        *reinterpret_cast<__nv_bfloat162*>(y + r1 * N + col) =
                            __floats2bfloat162_rn(acc[m][t][2] + b0, acc[m][t][3] + b1);
                }
            }
        }
    }
}

template <int K, int N, bool LN = false>
int rows_gemm_run(const void* x, const float* lnw, const float* lnb, float eps, const void* w, const float* bias,
                  void* y, int64_t M, cudaStream_t st) {
    using G = RgGeom<K, N>;
    constexpr size_t smem = LN ? G::kSmemLn : G::kSmem;
    const void* fn = reinterpret_cast<const void*>(&rows_gemm_kernel<K, N, LN>);
    if (!ensure_smem_attr(fn, smem))
        return fail(VH_E_DEVICE, "row gemm: cannot reserve %zu bytes of shared memory", smem);
    // Resident CTAs per SM of this instantiation, per device (GPUs of a process may differ);
    // concurrent first calls may both query it, and store the same value.
    static std::atomic<int> per_sm_cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    int per_sm = per_sm_cache[dev].load(std::memory_order_relaxed);
    if (per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kRgThreads, smem) != cudaSuccess || n <= 0) n = 1;
        per_sm = n;
        per_sm_cache[dev].store(n, std::memory_order_relaxed);
    }
    const int64_t tiles = (M + 15) / 16;
    const int64_t want = (tiles + kRgWarps - 1) / kRgWarps;
    const int grid = (int)std::min<int64_t>(want, (int64_t)per_sm * sm_count());
    rows_gemm_kernel<K, N, LN><<<grid, kRgThreads, smem, st>>>(x, lnw, lnb, eps, static_cast<const __nv_bfloat16*>(w),
                                                               bias, static_cast<__nv_bfloat16*>(y), M);
    return launch_status(LN ? "layernorm row gemm" : "row gemm");
}

template <int K>
int rows_gemm_n(int N, const void* x, const void* w, const float* bias, void* y, int64_t M, cudaStream_t st) {
    switch (N) {
        case 32: return rows_gemm_run<K, 32>(x, nullptr, nullptr, 0.f, w, bias, y, M, st);
        case 64: return rows_gemm_run<K, 64>(x, nullptr, nullptr, 0.f, w, bias, y, M, st);
        case 128: return rows_gemm_run<K, 128>(x, nullptr, nullptr, 0.f, w, bias, y, M, st);
        default: return rows_gemm_run<K, 256>(x, nullptr, nullptr, 0.f, w, bias, y, M, st);
    }
}

template <int K>
int ln_rows_gemm_n(int N, const float* x, const float* lnw, const float* lnb, float eps, const void* w,
                   const float* bias, void* y, int64_t M, cudaStream_t st) {
    return N == 32 ? rows_gemm_run<K, 32, true>(x, lnw, lnb, eps, w, bias, y, M, st)
                   : rows_gemm_run<K, 64, true>(x, lnw, lnb, eps, w, bias, y, M, st);
}

}  // namespace
}  // namespace vh

using namespace vh;

extern "C" int vh_rows_gemm_fwd(const void* x, const void* weight, const float* bias, void* y, int64_t rows,
                                int32_t in_features, int32_t out_features, vh_stream_t stream) {
    clear_error();
    if (!x || !weight || !y) return fail(VH_E_ARG, "vh_rows_gemm_fwd: null pointer argument");
    const int K = in_features, N = out_features;
    auto pow2_ok = [](int v) { return v == 32 || v == 64 || v == 128 || v == 256; };
    if (!pow2_ok(K) || !pow2_ok(N) || K * N > 32768)
        return fail(VH_E_SHAPE, "vh_rows_gemm_fwd: in/out features must be 32, 64, 128 or 256 with in*out <= 32768 "
                    "(got %d x %d)", K, N);
    if (rows <= 0) return fail(VH_E_SHAPE, "vh_rows_gemm_fwd: empty input");
    if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(y, 16) || (bias && !aligned(bias, 4)))
        return fail(VH_E_ALIGN, "vh_rows_gemm_fwd: misaligned pointers");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (K) {
        case 32: return rows_gemm_n<32>(N, x, weight, bias, y, rows, st);
        case 64: return rows_gemm_n<64>(N, x, weight, bias, y, rows, st);
        case 128: return rows_gemm_n<128>(N, x, weight, bias, y, rows, st);
        default: return rows_gemm_n<256>(N, x, weight, bias, y, rows, st);
    }
}

extern "C" int vh_ln_rows_gemm_fwd(const float* x, const float* ln_weight, const float* ln_bias, float eps,
                                   const void* weight, const float* bias, void* y, int64_t rows,
                                   int32_t in_features, int32_t out_features, vh_stream_t stream) {
    clear_error();
    if (!x || !ln_weight || !ln_bias || !weight || !y)
        return fail(VH_E_ARG, "vh_ln_rows_gemm_fwd: null pointer argument");
    const int K = in_features, N = out_features;
    if ((K != 32 && K != 64 && K != 128) || (N != 32 && N != 64))
        return fail(VH_E_SHAPE, "vh_ln_rows_gemm_fwd: in_features must be 32, 64 or 128 and out_features 32 or 64 "
                    "(got %d x %d)", K, N);
    if (rows <= 0) return fail(VH_E_SHAPE, "vh_ln_rows_gemm_fwd: empty input");
    if (!(eps >= 0.f)) return fail(VH_E_ARG, "vh_ln_rows_gemm_fwd: eps must be >= 0");
    if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(y, 16) || !aligned(ln_weight, 16) ||
        !aligned(ln_bias, 16) || (bias && !aligned(bias, 4)))
        return fail(VH_E_ALIGN, "vh_ln_rows_gemm_fwd: misaligned pointers");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (K) {
        case 32: return ln_rows_gemm_n<32>(N, x, ln_weight, ln_bias, eps, weight, bias, y, rows, st);
        case 64: return ln_rows_gemm_n<64>(N, x, ln_weight, ln_bias, eps, weight, bias, y, rows, st);
        default: return ln_rows_gemm_n<128>(N, x, ln_weight, ln_bias, eps, weight, bias, y, rows, st);
    }
}
