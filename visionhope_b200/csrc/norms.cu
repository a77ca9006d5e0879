// GRN and channel LayerNorm kernels on channels-last rows, fp32 output, with C entry points.
// Both are HBM-bound: every load/store is a 4-channel vector and grids cover all SMs.
#include <algorithm>
#include <mutex>
#include <set>
#include <tuple>
#include <type_traits>

#include "abi_util.h"
#include "common.cuh"

namespace vh {

// =============================== GRN (utils/csrc/grn_cuda.cu:46-124) ==========================
// Pass 1: per (b, pixel slice) partial sums of x^2 per channel -> workspace [B, splits, C].
// Pass 2: every CTA of (b, slice) folds the partials into Gx[c] = sqrt(sum), the per-image
//         1 / (mean_c Gx + eps), a per-channel factor f[c] = 1 + gamma[c] Gx[c] inv_den, and
//         writes y = x f[c] + beta[c] for its slice.
constexpr int kGrnThreads = 256;
constexpr int kGrnTargetCtas = 600;  // ~4 CTAs per SM on a 148-SM B200

inline int grn_splits(int B, int64_t S) {
    int64_t s = (kGrnTargetCtas + B - 1) / B;
    s = std::min<int64_t>(s, std::max<int64_t>(1, S / 8));
    return (int)std::max<int64_t>(1, std::min<int64_t>(s, 1024));
}

template <typename T>
__global__ void __launch_bounds__(kGrnThreads) grn_stats_kernel(const T* __restrict__ x,
                                                                float* __restrict__ part, int C,
                                                                int64_t S, int splits) {
    extern __shared__ float red[];  // [rphases][Geff * 4]
    const int b = blockIdx.y, split = blockIdx.x;
    const int G = C / 4;
    const int Geff = min(G, kGrnThreads);
    const int rph = kGrnThreads / Geff;
    const int gi = threadIdx.x % Geff, ri = threadIdx.x / Geff;
    const int64_t s0 = S * split / splits, s1 = S * (split + 1) / splits;
    const T* xb = x + (int64_t)b * S * C;
    for (int gb = 0; gb < G; gb += Geff) {
        const int g = gb + gi;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ri < rph && g < G) {
            for (int64_t s = s0 + ri; s < s1; s += rph) {
                const float4 v = load4(xb + s * C + 4 * g);
                acc.x = fmaf(v.x, v.x, acc.x);
                acc.y = fmaf(v.y, v.y, acc.y);
                acc.z = fmaf(v.z, v.z, acc.z);
                acc.w = fmaf(v.w, v.w, acc.w);
            }
        }
        if (ri < rph) {
            float* r = red + ((size_t)ri * Geff + gi) * 4;
            r[0] = acc.x; r[1] = acc.y; r[2] = acc.z; r[3] = acc.w;
        }
        __syncthreads();
        for (int it = threadIdx.x; it < Geff * 4; it += blockDim.x) {
            const int cg = gb * 4 + it;
            float sum = 0.f;
            for (int k = 0; k < rph; ++k) sum += red[(size_t)k * Geff * 4 + it];
            if (cg < C) part[((int64_t)b * splits + split) * C + cg] = sum;
        }
        __syncthreads();
    }
}

template <typename T, typename YT = float>
__global__ void __launch_bounds__(kGrnThreads) grn_apply_kernel(
    const T* __restrict__ x, const float* __restrict__ part, const float* __restrict__ gamma,
    const float* __restrict__ beta, float eps, YT* __restrict__ y, float* __restrict__ gx_out,
    float* __restrict__ inv_out, int C, int64_t S, int splits) {
    extern __shared__ float fac[];  // [C] factors, then [32] reduction scratch
    float* scratch = fac + C;
    const int b = blockIdx.y, split = blockIdx.x;
    const float* pb = part + (int64_t)b * splits * C;
    float local = 0.f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float s = 0.f;
        for (int k = 0; k < splits; ++k) s += pb[(int64_t)k * C + c];
        const float g = sqrtf(s);
        fac[c] = g;
        local += g;
    }
    local = warp_sum(local);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? scratch[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) scratch[0] = 1.f / (v / (float)C + eps);
    }
    __syncthreads();
    const float inv_den = scratch[0];
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float g = fac[c];
        if (split == 0 && gx_out) gx_out[(int64_t)b * C + c] = g;
        fac[c] = 1.f + gamma[c] * (g * inv_den);
    }
    if (split == 0 && inv_out && threadIdx.x == 0) inv_out[b] = inv_den;
    __syncthreads();
    const int G = C / 4;
    const int64_t s0 = S * split / splits, s1 = S * (split + 1) / splits;
    const int64_t n = (s1 - s0) * G;
    const T* xb = x + ((int64_t)b * S + s0) * C;
    YT* yb = y + ((int64_t)b * S + s0) * C;
    for (int64_t it = threadIdx.x; it < n; it += blockDim.x) {
        const int64_t s = it / G;
        const int c = (int)(it % G) * 4;
        const float4 v = load4(xb + s * C + c);
        float4 o;
        o.x = fmaf(v.x, fac[c + 0], beta[c + 0]);
        o.y = fmaf(v.y, fac[c + 1], beta[c + 1]);
        o.z = fmaf(v.z, fac[c + 2], beta[c + 2]);
        o.w = fmaf(v.w, fac[c + 3], beta[c + 3]);
        store4(yb + s * C + c, o);
    }
}

// ====== GRN from precomputed sums of squares (the statistics pass fused into the producer) =====
// part [B, nparts, C]: sums of x^2 per channel over disjoint pixel slices of each image (the
// FFN's depthwise GELU kernel writes them per pixel tile as it stores x).
// grn_factor_kernel: one CTA per image sums the slices in index order and writes the factors
//   f[b, c] = 1 + gamma[c] Gx[c] / (mean_c Gx + eps), Gx = sqrt(sum)  (as grn_apply_kernel).
// grn_scale8_kernel: y = x f[b, c] + beta[c] over all 16-byte vectors of the batch, a grid of
//   a few CTAs per SM striding over them; a CTA has C / 8 x floor(256 / (C / 8)) threads, so
//   the stride is a multiple of C / 8 and each thread keeps one channel group (its betas in
//   registers); four vector loads are in flight before any is used.  Needs C % 8 == 0 and
//   C <= 2048.
constexpr int kGrnScaleUnroll = 4;
// CTAs per SM: 16-bit x loads its factors together with x (3 CTAs, registers for both); fp32 x
// (twice the registers per vector) reads them after its x loads, at 4 CTAs.
template <typename T>
constexpr int grn_scale_ctas_per_sm() { return sizeof(T) == 4 ? 4 : 3; }

// A thread owns the channels tid, tid + 256, ... (at most kGrnFactorCh of them: C <= 2048) and
// keeps their sums in registers from the one pass over the slices: the loads of kGrnFactorK
// slices for all its channels are issued before any is added, and each channel still sums its
// slices in index order.
constexpr int kGrnFactorCh = 8;
constexpr int kGrnFactorK = 4;

__global__ void __launch_bounds__(kGrnThreads) grn_factor_kernel(const float* __restrict__ part, int nparts,
                                                                 const float* __restrict__ gamma, float eps,
                                                                 float* __restrict__ fac_out, int C) {
    __shared__ float scratch[32];
    const int b = blockIdx.x;
    const float* pb = part + (int64_t)b * nparts * C;
    float s[kGrnFactorCh];
#pragma unroll
    for (int j = 0; j < kGrnFactorCh; ++j) s[j] = 0.f;
    for (int k0 = 0; k0 < nparts; k0 += kGrnFactorK) {
        float v[kGrnFactorK][kGrnFactorCh];
#pragma unroll
        for (int k = 0; k < kGrnFactorK; ++k)
#pragma unroll
            for (int j = 0; j < kGrnFactorCh; ++j) {
                const int c = threadIdx.x + j * kGrnThreads;
                v[k][j] = (k0 + k < nparts && c < C) ? pb[(int64_t)(k0 + k) * C + c] : 0.f;
            }
#pragma unroll
        for (int k = 0; k < kGrnFactorK; ++k)
#pragma unroll
            for (int j = 0; j < kGrnFactorCh; ++j)
                if (k0 + k < nparts) s[j] += v[k][j];
    }
    float local = 0.f;
#pragma unroll
    for (int j = 0; j < kGrnFactorCh; ++j) {
        s[j] = sqrtf(s[j]);  // Gx of this thread's channel j
        if (threadIdx.x + j * kGrnThreads < C) local += s[j];
    }
    local = warp_sum(local);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? scratch[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) scratch[0] = 1.f / (v / (float)C + eps);
    }
    __syncthreads();
    const float inv_den = scratch[0];
#pragma unroll
    for (int j = 0; j < kGrnFactorCh; ++j) {
        const int c = threadIdx.x + j * kGrnThreads;
        if (c < C) fac_out[(int64_t)b * C + c] = 1.f + gamma[c] * (s[j] * inv_den);
    }
}

template <typename T, typename YT>
__global__ void __launch_bounds__(kGrnThreads, grn_scale_ctas_per_sm<T>()) grn_scale8_kernel(
    const T* __restrict__ x, const float* __restrict__ fac, const float* __restrict__ beta,
    YT* __restrict__ y, int C, uint32_t per_image, uint32_t nvec) {
    const uint32_t G8 = (uint32_t)C >> 3, stride = gridDim.x * blockDim.x;
    const uint32_t v0 = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = 8 * (int)(v0 % G8);
    float bt[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) bt[e] = beta[c + e];
    for (uint32_t v = v0; v < nvec; v += stride * kGrnScaleUnroll) {
        // 16-bit x: the factors of each vector are loaded with it, so neither waits for the other.
        constexpr bool kEarly = sizeof(T) != 4;
        uint4 raw[kGrnScaleUnroll][sizeof(T) == 4 ? 2 : 1];
        float4 fa[kEarly ? kGrnScaleUnroll : 1], fb[kEarly ? kGrnScaleUnroll : 1];
#pragma unroll
        for (int u = 0; u < kGrnScaleUnroll; ++u) {
            const uint32_t vu = v + u * stride;
            if (vu < nvec) {
                const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)vu * 8);
#pragma unroll
                for (int h = 0; h < (sizeof(T) == 4 ? 2 : 1); ++h) raw[u][h] = __ldcs(src + h);
                if constexpr (kEarly) {
                    const float* f = fac + (size_t)(vu / per_image) * C + c;
                    fa[u] = *reinterpret_cast<const float4*>(f);
                    fb[u] = *reinterpret_cast<const float4*>(f + 4);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kGrnScaleUnroll; ++u) {
            const uint32_t vu = v + u * stride;
            if (vu >= nvec) break;
            float4 f0, f1;
            if constexpr (kEarly) {
                f0 = fa[u];
                f1 = fb[u];
            } else {
                const float* f = fac + (size_t)(vu / per_image) * C + c;
                f0 = *reinterpret_cast<const float4*>(f);
                f1 = *reinterpret_cast<const float4*>(f + 4);
            }
            float xv[8];
            load8(reinterpret_cast<const T*>(&raw[u][0]), xv);
            const float fv[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) xv[e] = fmaf(xv[e], fv[e], bt[e]);
            store8(y + (size_t)vu * 8, xv);
        }
    }
}

// ============ GRN in one read: a thread-block cluster per image (grn_cuda.cu:46-124) ============
// The K CTAs of image b each copy a contiguous slice of its pixels (all channels) into shared
// memory with asynchronous 16-byte copies, sum x^2 per channel over the slice, and read the K
// partial sums of every channel from the cluster's shared memory.  Each CTA then forms
// Gx = sqrt(sum), inv_den = 1 / (mean_c Gx + eps) and f[c] = 1 + gamma[c] Gx[c] inv_den, and
// writes y = x f[c] + beta[c] from its resident slice: x is read from HBM once.
constexpr int kGrnClusterMax = 16;

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;\n" : "=r"(r));
    return r;
}
// Reads a float at the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// Shared memory: part[C], fac[C], beta[C], red[4 * kGrnThreads], scratch[32], then the slice.
__host__ __device__ inline size_t grn_cluster_head_bytes(int C) {
    return ((size_t)3 * C * 4 + 4 * kGrnThreads * 4 + 32 * 4 + 15) & ~size_t(15);
}

template <typename T, typename YT>
__global__ void __launch_bounds__(kGrnThreads) grn_cluster_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
    YT* __restrict__ y, float* __restrict__ gx_out, float* __restrict__ inv_out, int C, int S) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* part = reinterpret_cast<float*>(smem);
    float* fac = part + C;
    float* bet = fac + C;
    float* red = bet + C;
    float* scratch = red + 4 * kGrnThreads;
    T* xs = reinterpret_cast<T*>(smem + grn_cluster_head_bytes(C));
    const uint32_t K = cluster_size(), rank = cluster_rank();
    const int b = blockIdx.y, tid = threadIdx.x;
    const int s0 = (int)((int64_t)S * rank / K), s1 = (int)((int64_t)S * (rank + 1) / K);
    const int rows = s1 - s0;

    // 1. the slice [s0, s1) x C is contiguous: asynchronous 16-byte copies, all in flight.
    {
        const char* src = reinterpret_cast<const char*>(x + ((int64_t)b * S + s0) * C);
        char* dst = reinterpret_cast<char*>(xs);
        const int nvec = (int)((int64_t)rows * C * (int)sizeof(T) / 16);
        for (int i = tid; i < nvec; i += kGrnThreads) cp_async<16>(dst + 16 * (size_t)i, src + 16 * (size_t)i);
        cp_async_commit();
    }
    for (int c = tid; c < C; c += kGrnThreads) bet[c] = beta[c];
    cp_async_wait<0>();
    __syncthreads();

    // 2. per-channel sums of squares over the slice; thread (qi, ri) owns channel quad qi and
    //    the pixel phase ri (rph phases).
    const int Q = C / 4;
    for (int q0 = 0; q0 < Q; q0 += kGrnThreads) {
        const int qn = min(Q - q0, kGrnThreads), rph = kGrnThreads / qn;
        const int qi = tid % qn, ri = tid / qn;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ri < rph) {
            for (int r = ri; r < rows; r += rph) {
                const float4 v = load4(xs + (size_t)r * C + 4 * (q0 + qi));
                acc.x = fmaf(v.x, v.x, acc.x);
                acc.y = fmaf(v.y, v.y, acc.y);
                acc.z = fmaf(v.z, v.z, acc.z);
                acc.w = fmaf(v.w, v.w, acc.w);
            }
            *reinterpret_cast<float4*>(red + 4 * (ri * qn + qi)) = acc;
        }
        __syncthreads();
        for (int it = tid; it < qn * 4; it += kGrnThreads) {
            float sum = 0.f;
            for (int k = 0; k < rph; ++k) sum += red[k * qn * 4 + it];
            part[q0 * 4 + it] = sum;
        }
        __syncthreads();
    }

    // 3. exchange the partial sums across the cluster.
    cluster_arrive();
    cluster_wait();
    float local = 0.f;
    for (int c = tid; c < C; c += kGrnThreads) {
        float sum = 0.f;
        for (uint32_t k = 0; k < K; ++k) sum += ld_cluster_f32(part + c, k);
        const float g = sqrtf(sum);
        fac[c] = g;
        local += g;
    }
    cluster_arrive();  // this CTA has finished reading the others' partial sums
    local = warp_sum(local);
    if ((tid & 31) == 0) scratch[tid >> 5] = local;
    __syncthreads();
    if (tid < 32) {
        float v = tid < kGrnThreads / 32 ? scratch[tid] : 0.f;
        v = warp_sum(v);
        if (tid == 0) scratch[0] = 1.f / (v / (float)C + eps);
    }
    __syncthreads();
    const float inv_den = scratch[0];
    for (int c = tid; c < C; c += kGrnThreads) {
        const float g = fac[c];
        if (rank == 0 && gx_out) gx_out[(int64_t)b * C + c] = g;
        fac[c] = 1.f + gamma[c] * (g * inv_den);
    }
    if (rank == 0 && inv_out && tid == 0) inv_out[b] = inv_den;
    __syncthreads();

    // 4. y = x f + beta from the resident slice.
    YT* dst = y + ((int64_t)b * S + s0) * C;
    for (int q0 = 0; q0 < Q; q0 += kGrnThreads) {
        const int qn = min(Q - q0, kGrnThreads), rph = kGrnThreads / qn;
        const int qi = tid % qn, ri = tid / qn;
        if (ri >= rph) continue;
        const int c = 4 * (q0 + qi);
        const float4 f = *reinterpret_cast<const float4*>(fac + c);
        const float4 be = *reinterpret_cast<const float4*>(bet + c);
        for (int r = ri; r < rows; r += rph) {
            const float4 v = load4(xs + (size_t)r * C + c);
            store4(dst + (size_t)r * C + c,
                   make_float4(fmaf(v.x, f.x, be.x), fmaf(v.y, f.y, be.y), fmaf(v.z, f.z, be.z), fmaf(v.w, f.w, be.w)));
        }
    }
    cluster_wait();  // no CTA leaves while another may still read its partial sums
}

// ====================== LayerNorm over channels (layer_norm_cuda.py:31-57) ======================
// SW lanes per row (SW in {8, 16, 32}), each lane holds NV 4-channel vectors in registers;
// mean and biased variance by two in-register passes (the Triton kernel's order).
constexpr int kLnThreads = 256;

template <typename T, typename YT, int SW, int NV>
__global__ void __launch_bounds__(kLnThreads) ln_kernel(const T* __restrict__ x,
                                                        const float* __restrict__ w,
                                                        const float* __restrict__ bias, float eps,
                                                        YT* __restrict__ y, float* __restrict__ mean_out,
                                                        float* __restrict__ rstd_out, int64_t rows, int C) {
    const int lane = threadIdx.x % SW;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / SW;
    const unsigned mask = SW == 32 ? 0xffffffffu : (((1u << SW) - 1u) << ((threadIdx.x & 31) & ~(SW - 1)));
    const bool live = row < rows;
    const int G = C / 4;
    const T* xr = x + (live ? row : 0) * C;
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int g = lane + k * SW;
        if (live && g < G) {
            v[k] = load4(xr + 4 * g);
            s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        } else {
            v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
#pragma unroll
    for (int o = SW / 2; o > 0; o >>= 1) s += __shfl_xor_sync(mask, s, o, SW);
    const float mean = s / (float)C;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int g = lane + k * SW;
        if (g < G) {
            const float a = v[k].x - mean, b2 = v[k].y - mean, c2 = v[k].z - mean, d = v[k].w - mean;
            q += (a * a + b2 * b2) + (c2 * c2 + d * d);
        }
    }
#pragma unroll
    for (int o = SW / 2; o > 0; o >>= 1) q += __shfl_xor_sync(mask, q, o, SW);
    const float rstd = 1.f / sqrtf(q / (float)C + eps);
    if (!live) return;
    YT* yr = y + row * C;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int g = lane + k * SW;
        if (g < G) {
            const int c = 4 * g;
            float4 o;
            o.x = (v[k].x - mean) * rstd * w[c + 0] + bias[c + 0];
            o.y = (v[k].y - mean) * rstd * w[c + 1] + bias[c + 1];
            o.z = (v[k].z - mean) * rstd * w[c + 2] + bias[c + 2];
            o.w = (v[k].w - mean) * rstd * w[c + 3] + bias[c + 3];
            store4(yr + c, o);
        }
    }
    if (lane == 0) {
        if (mean_out) mean_out[row] = mean;
        if (rstd_out) rstd_out[row] = rstd;
    }
}

// Residual operand type of ln8_kernel when there is no residual add.
struct NoResidual {};

// C a multiple of 8: SW lanes per row, each lane holds NV 8-channel vectors of R rows in
// registers (all R * NV 16-byte loads are issued before any arithmetic), so enough bytes are
// in flight per SM to run at HBM speed.  Same two in-register passes as ln_kernel.  With a
// residual operand (RT not NoResidual) each row is first replaced by s = x + r, stored to
// sum_out in x's dtype (sum_out may be x), and normalized as stored.
template <typename T, typename YT, int SW, int NV, int R, typename RT = NoResidual>
__global__ void __launch_bounds__(kLnThreads) ln8_kernel(const T* x, const RT* __restrict__ radd, T* sum_out,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ bias, float eps,
                                                         YT* __restrict__ y, float* __restrict__ mean_out,
                                                         float* __restrict__ rstd_out, int64_t rows, int C) {
    constexpr int GPC = kLnThreads / SW;  // row groups per CTA
    const int lane = threadIdx.x % SW, grp = threadIdx.x / SW;
    const int64_t base = (int64_t)blockIdx.x * GPC * R + grp;
    const int G8 = C / 8;
    float v[R][NV][8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t row = base + (int64_t)r * GPC;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int g = lane + k * SW;
            if (row < rows && g < G8) {
                load8(x + row * C + 8 * g, v[r][k]);
                if constexpr (!std::is_same<RT, NoResidual>::value) {
                    float rv[8];
                    load8(radd + row * C + 8 * g, rv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[r][k][e] += rv[e];
                    store8(sum_out + row * C + 8 * g, v[r][k]);
                    if constexpr (!std::is_same<T, float>::value) {
                        load8(sum_out + row * C + 8 * g, v[r][k]);  // normalize s as stored
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[r][k][e] = 0.f;
            }
        }
    }
    const float invC = 1.f / (float)C;
    float mean[R], rstd[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k)
            s += ((v[r][k][0] + v[r][k][1]) + (v[r][k][2] + v[r][k][3])) +
                 ((v[r][k][4] + v[r][k][5]) + (v[r][k][6] + v[r][k][7]));
#pragma unroll
        for (int o = SW / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o, SW);
        mean[r] = s / (float)C;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int g = lane + k * SW;
            if (g < G8) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float d = v[r][k][e] - mean[r];
                    q = fmaf(d, d, q);
                }
            }
        }
#pragma unroll
        for (int o = SW / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o, SW);
        rstd[r] = 1.f / sqrtf(q * invC + eps);
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int g = lane + k * SW;
        if (g >= G8) continue;
        float wv[8], bv[8];
        load8(w + 8 * g, wv);
        load8(bias + 8 * g, bv);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t row = base + (int64_t)r * GPC;
            if (row >= rows) continue;
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = (v[r][k][e] - mean[r]) * rstd[r] * wv[e] + bv[e];
            store8(y + row * C + 8 * g, o);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t row = base + (int64_t)r * GPC;
            if (row >= rows) continue;
            if (mean_out) mean_out[row] = mean[r];
            if (rstd_out) rstd_out[row] = rstd[r];
        }
    }
}

// Any C: one warp per row, scalar accesses, two passes over global memory.
template <typename T, typename YT>
__global__ void __launch_bounds__(kLnThreads) ln_generic_kernel(const T* __restrict__ x,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ bias, float eps,
                                                                YT* __restrict__ y,
                                                                float* __restrict__ mean_out,
                                                                float* __restrict__ rstd_out,
                                                                int64_t rows, int C) {
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const T* xr = x + row * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += to_f(xr[c]);
    s = warp_sum(s);
    const float mean = s / (float)C;
    float q = 0.f;
    for (int c = lane; c < C; c += 32) {
        const float a = to_f(xr[c]) - mean;
        q += a * a;
    }
    q = warp_sum(q);
    const float rstd = 1.f / sqrtf(q / (float)C + eps);
    YT* yr = y + row * C;
    for (int c = lane; c < C; c += 32) yr[c] = from_f<YT>((to_f(xr[c]) - mean) * rstd * w[c] + bias[c]);
    if (lane == 0) {
        if (mean_out) mean_out[row] = mean;
        if (rstd_out) rstd_out[row] = rstd;
    }
}

// Cluster size for the single-read GRN, or 0 when the two-pass form must be used: the
// smallest K <= 16 whose per-CTA slice fits 110 KB (two CTAs per SM), else 200 KB.
template <typename T>
int grn_cluster_plan(const void* x, int64_t S, int C, size_t* smem_out) {
    if (S > (1 << 30) || ((size_t)C * sizeof(T)) % 16 || !aligned(x, 16)) return 0;
    const size_t head = grn_cluster_head_bytes(C);
    for (size_t budget : {(size_t)110 * 1024, (size_t)200 * 1024}) {
        for (int K = 1; K <= kGrnClusterMax; ++K) {
            const size_t smem = head + (size_t)((S + K - 1) / K) * C * sizeof(T);
            if (smem <= budget) {
                *smem_out = smem;
                return K;
            }
        }
    }
    return 0;
}

// Whether a cluster of K CTAs with `smem` bytes each can be resident (queried once per shape).
template <typename T, typename YT>
bool grn_cluster_ok(int K, size_t smem) {
    static std::mutex mu;
    static std::set<std::tuple<int, int, size_t>> good, bad;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const auto key = std::make_tuple(dev, K, smem);
    std::lock_guard<std::mutex> lock(mu);
    if (good.count(key)) return true;
    if (bad.count(key)) return false;
    const void* fn = reinterpret_cast<const void*>(&grn_cluster_kernel<T, YT>);
    bool ok = ensure_smem_attr(fn, smem);
    if (ok && K > 8) ok = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
    if (ok) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(K, 1, 1);
        cfg.blockDim = dim3(kGrnThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = K;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        ok = cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) == cudaSuccess && clusters > 0;
    }
    cudaGetLastError();  // a refused query leaves no sticky error behind
    (ok ? good : bad).insert(key);
    return ok;
}

template <typename T, typename YT>
int grn_run(const void* xv, const float* gamma, const float* beta, float eps, YT* y, float* gx,
            float* inv, float* part, int B, int64_t S, int C, cudaStream_t st) {
    const T* x = static_cast<const T*>(xv);
    size_t csmem = 0;
    const int K = aligned(y, 8 * sizeof(YT) / 2) ? grn_cluster_plan<T>(xv, S, C, &csmem) : 0;
    if (K > 0 && grn_cluster_ok<T, YT>(K, csmem)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(K, B, 1);
        cfg.blockDim = dim3(kGrnThreads, 1, 1);
        cfg.dynamicSmemBytes = csmem;
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = K;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, grn_cluster_kernel<T, YT>, x, gamma, beta, eps, y, gx, inv, C, (int)S);
        return launch_status("grn (cluster)");
    }
    const int splits = grn_splits(B, S);
    const int G = C / 4;
    const int Geff = std::min(G, kGrnThreads);
    const int rph = kGrnThreads / Geff;
    const size_t red_bytes = sizeof(float) * (size_t)rph * Geff * 4;
    dim3 grid(splits, B);
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&grn_stats_kernel<T>), red_bytes))
        return fail(VH_E_DEVICE, "grn: shared memory");
    grn_stats_kernel<T><<<grid, kGrnThreads, red_bytes, st>>>(x, part, C, S, splits);
    int rc = launch_status("grn stats");
    if (rc) return rc;
    const size_t fac_bytes = sizeof(float) * ((size_t)C + 32);
    if (!ensure_smem_attr(reinterpret_cast<const void*>(&grn_apply_kernel<T, YT>), fac_bytes))
        return fail(VH_E_DEVICE, "grn: shared memory");
    grn_apply_kernel<T, YT><<<grid, kGrnThreads, fac_bytes, st>>>(x, part, gamma, beta, eps, y, gx, inv, C,
                                                                   S, splits);
    return launch_status("grn apply");
}

template <typename T>
int grn_run_y(int y_dtype, const void* xv, const float* gamma, const float* beta, float eps, void* y,
              float* gx, float* inv, float* part, int B, int64_t S, int C, cudaStream_t st) {
    switch (y_dtype) {
        case VH_F32: return grn_run<T, float>(xv, gamma, beta, eps, static_cast<float*>(y), gx, inv, part, B, S, C, st);
        case VH_BF16: return grn_run<T, __nv_bfloat16>(xv, gamma, beta, eps, static_cast<__nv_bfloat16*>(y), gx, inv, part, B, S, C, st);
        default: return grn_run<T, __half>(xv, gamma, beta, eps, static_cast<__half*>(y), gx, inv, part, B, S, C, st);
    }
}

template <typename T, typename YT, int SW, int NV>
int ln_launch(const void* x, const float* w, const float* b, float eps, YT* y, float* m, float* r,
              int64_t rows, int C, cudaStream_t st) {
    const int64_t rows_per_cta = kLnThreads / SW;
    const int64_t blocks = (rows + rows_per_cta - 1) / rows_per_cta;
    ln_kernel<T, YT, SW, NV><<<(unsigned)blocks, kLnThreads, 0, st>>>(static_cast<const T*>(x), w, b, eps, y,
                                                                      m, r, rows, C);
    return launch_status("layernorm");
}

template <typename T, typename YT, int SW, int NV, int R>
int ln8_launch(const void* x, const float* w, const float* b, float eps, YT* y, float* m, float* r,
               int64_t rows, int C, cudaStream_t st) {
    const int64_t rows_per_cta = (int64_t)(kLnThreads / SW) * R;
    const int64_t blocks = (rows + rows_per_cta - 1) / rows_per_cta;
    ln8_kernel<T, YT, SW, NV, R><<<(unsigned)blocks, kLnThreads, 0, st>>>(
        static_cast<const T*>(x), static_cast<const NoResidual*>(nullptr), static_cast<T*>(nullptr), w, b, eps,
        y, m, r, rows, C);
    return launch_status("layernorm");
}

template <typename T, typename RT, typename YT, int SW, int NV, int R>
int add_ln8_launch(const void* x, const void* radd, void* sum_out, const float* w, const float* b, float eps,
                   YT* y, int64_t rows, int C, cudaStream_t st) {
    const int64_t rows_per_cta = (int64_t)(kLnThreads / SW) * R;
    const int64_t blocks = (rows + rows_per_cta - 1) / rows_per_cta;
    ln8_kernel<T, YT, SW, NV, R, RT><<<(unsigned)blocks, kLnThreads, 0, st>>>(
        static_cast<const T*>(x), static_cast<const RT*>(radd), static_cast<T*>(sum_out), w, b, eps, y, nullptr,
        nullptr, rows, C);
    return launch_status("add layernorm");
}

// Residual add + LayerNorm, C a multiple of 8 (checked by the entry point).
template <typename T, typename RT, typename YT>
int add_ln_run(const void* x, const void* radd, void* sum_out, const float* w, const float* b, float eps, YT* y,
               int64_t rows, int C, cudaStream_t st) {
    const int G8 = C / 8;
    if (G8 <= 4) return add_ln8_launch<T, RT, YT, 4, 1, 4>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    if (G8 <= 8) return add_ln8_launch<T, RT, YT, 8, 1, 4>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    if (G8 <= 16) return add_ln8_launch<T, RT, YT, 16, 1, 2>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    if (G8 <= 32) return add_ln8_launch<T, RT, YT, 32, 1, 2>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    if (G8 <= 64) return add_ln8_launch<T, RT, YT, 32, 2, 2>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    if (G8 <= 128) return add_ln8_launch<T, RT, YT, 32, 4, 1>(x, radd, sum_out, w, b, eps, y, rows, C, st);
    return add_ln8_launch<T, RT, YT, 32, 8, 1>(x, radd, sum_out, w, b, eps, y, rows, C, st);
}

template <typename T, typename RT>
int add_ln_y(int y_dtype, const void* x, const void* radd, void* sum_out, const float* w, const float* b,
             float eps, void* y, int64_t rows, int C, cudaStream_t st) {
    switch (y_dtype) {
        case VH_F32: return add_ln_run<T, RT, float>(x, radd, sum_out, w, b, eps, static_cast<float*>(y), rows, C, st);
        case VH_BF16: return add_ln_run<T, RT, __nv_bfloat16>(x, radd, sum_out, w, b, eps, static_cast<__nv_bfloat16*>(y), rows, C, st);
        default: return add_ln_run<T, RT, __half>(x, radd, sum_out, w, b, eps, static_cast<__half*>(y), rows, C, st);
    }
}

template <typename T, typename YT>
int ln_run(const void* x, const float* w, const float* b, float eps, YT* y, float* m, float* r,
           int64_t rows, int C, bool vec_ok, cudaStream_t st) {
    const int G = C / 4;
    const bool vec8 = C % 8 == 0 && aligned(x, 16) && aligned(y, 16) && aligned(w, 16) && aligned(b, 16);
    if (vec8) {
        const int G8 = C / 8;
        if (G8 <= 4) return ln8_launch<T, YT, 4, 1, 4>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 8) return ln8_launch<T, YT, 8, 1, 4>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 16) return ln8_launch<T, YT, 16, 1, 2>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 32) return ln8_launch<T, YT, 32, 1, 2>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 64) return ln8_launch<T, YT, 32, 2, 2>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 128) return ln8_launch<T, YT, 32, 4, 1>(x, w, b, eps, y, m, r, rows, C, st);
        if (G8 <= 256) return ln8_launch<T, YT, 32, 8, 1>(x, w, b, eps, y, m, r, rows, C, st);
    }
    if (vec_ok && C % 4 == 0) {
        if (G <= 8) return ln_launch<T, YT, 8, 1>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 16) return ln_launch<T, YT, 16, 1>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 32) return ln_launch<T, YT, 32, 1>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 64) return ln_launch<T, YT, 32, 2>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 128) return ln_launch<T, YT, 32, 4>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 256) return ln_launch<T, YT, 32, 8>(x, w, b, eps, y, m, r, rows, C, st);
        if (G <= 512) return ln_launch<T, YT, 32, 16>(x, w, b, eps, y, m, r, rows, C, st);
    }
    const int64_t blocks = (rows * 32 + kLnThreads - 1) / kLnThreads;
    ln_generic_kernel<T, YT><<<(unsigned)blocks, kLnThreads, 0, st>>>(static_cast<const T*>(x), w, b, eps, y,
                                                                      m, r, rows, C);
    return launch_status("layernorm");
}

template <typename T>
int ln_run_y(int y_dtype, const void* x, const float* w, const float* b, float eps, void* y, float* m,
             float* r, int64_t rows, int C, bool vec_ok, cudaStream_t st) {
    switch (y_dtype) {
        case VH_F32: return ln_run<T, float>(x, w, b, eps, static_cast<float*>(y), m, r, rows, C, vec_ok, st);
        case VH_BF16: return ln_run<T, __nv_bfloat16>(x, w, b, eps, static_cast<__nv_bfloat16*>(y), m, r, rows, C, vec_ok, st);
        default: return ln_run<T, __half>(x, w, b, eps, static_cast<__half*>(y), m, r, rows, C, vec_ok, st);
    }
}

}  // namespace vh

using namespace vh;

namespace vh {
int init_norm_kernels() { return 0; }
}  // namespace vh

extern "C" int64_t vh_grn_workspace_bytes(int32_t batch, int32_t height, int32_t width,
                                          int32_t channels) {
    if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0) return 0;
    const int64_t S = (int64_t)height * width;
    return (int64_t)sizeof(float) * batch * grn_splits(batch, S) * channels;
}

extern "C" int vh_grn_fwd(const void* x, int32_t x_dtype, const float* gamma, const float* beta,
                          float eps, void* y, int32_t y_dtype, float* gx, float* inv_den, void* workspace,
                          int64_t workspace_bytes, int32_t batch, int32_t height, int32_t width,
                          int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!x || !gamma || !beta || !y || !workspace) return fail(VH_E_ARG, "vh_grn_fwd: null pointer argument");
    if (!dtype_ok(x_dtype)) return fail(VH_E_DTYPE, "GRN supports FP32, FP16 and BF16 input");
    if (!dtype_ok(y_dtype)) return fail(VH_E_DTYPE, "vh_grn_fwd: bad output dtype");
    if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0)
        return fail(VH_E_SHAPE, "GRN expects nonempty input");
    if (channels % 4) return fail(VH_E_SHAPE, "vh_grn_fwd: channels must be a multiple of 4");
    if (batch > 65535) return fail(VH_E_RANGE, "vh_grn_fwd: batch must be <= 65535");
    if (!aligned(x, x_dtype == VH_F32 ? 16 : 8) || !aligned(y, y_dtype == VH_F32 ? 16 : 8) ||
        !aligned(workspace, 16))
        return fail(VH_E_ALIGN, "vh_grn_fwd: misaligned pointers");
    if (workspace_bytes < vh_grn_workspace_bytes(batch, height, width, channels))
        return fail(VH_E_ARG, "vh_grn_fwd: workspace too small (%lld < %lld bytes)",
                    (long long)workspace_bytes,
                    (long long)vh_grn_workspace_bytes(batch, height, width, channels));
    if ((size_t)channels * 4 + 128 > 200 * 1024) return fail(VH_E_RANGE, "vh_grn_fwd: too many channels");
    const int64_t S = (int64_t)height * width;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    switch (x_dtype) {
        case VH_F32: return grn_run_y<float>(y_dtype, x, gamma, beta, eps, y, gx, inv_den, part, batch, S, channels, st);
        case VH_BF16: return grn_run_y<__nv_bfloat16>(y_dtype, x, gamma, beta, eps, y, gx, inv_den, part, batch, S, channels, st);
        default: return grn_run_y<__half>(y_dtype, x, gamma, beta, eps, y, gx, inv_den, part, batch, S, channels, st);
    }
}

extern "C" int vh_grn_apply_fwd(const void* x, int32_t x_dtype, const float* sumsq, int32_t nparts,
                                const float* gamma, const float* beta, float eps, float* factors, void* y,
                                int32_t y_dtype, int32_t batch, int32_t height, int32_t width,
                                int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!x || !sumsq || !gamma || !beta || !factors || !y)
        return fail(VH_E_ARG, "vh_grn_apply_fwd: null pointer argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(VH_E_DTYPE, "vh_grn_apply_fwd: bad dtype");
    if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || nparts <= 0)
        return fail(VH_E_SHAPE, "GRN expects nonempty input");
    if (batch > 65535) return fail(VH_E_RANGE, "vh_grn_apply_fwd: batch must be <= 65535");
    if (channels % 8 || channels > 2048)
        return fail(VH_E_SHAPE, "vh_grn_apply_fwd: channels must be a multiple of 8, at most 2048");
    const int64_t per_image = (int64_t)height * width * (channels / 8);
    if (per_image * batch >= ((int64_t)1 << 32) - (int64_t)kGrnThreads * 1024 * kGrnScaleUnroll * 2)
        return fail(VH_E_RANGE, "vh_grn_apply_fwd: tensor too large");
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(factors, 16))
        return fail(VH_E_ALIGN, "vh_grn_apply_fwd: misaligned pointers");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    grn_factor_kernel<<<batch, kGrnThreads, 0, st>>>(sumsq, nparts, gamma, eps, factors, channels);
    int rc = launch_status("grn factors");
    if (rc) return rc;
    const uint32_t nvec = (uint32_t)(per_image * batch);
    const int threads = (channels / 8) * (kGrnThreads / (channels / 8));
    const int64_t want = (nvec + threads - 1) / threads;
    auto run = [&](auto xt, auto yt) -> int {
        using T = decltype(xt);
        using YT = decltype(yt);
        const dim3 grid((unsigned)std::min<int64_t>(want, (int64_t)sm_count() * grn_scale_ctas_per_sm<T>()));
        grn_scale8_kernel<T, YT><<<grid, threads, 0, st>>>(static_cast<const T*>(x), factors, beta,
                                                               static_cast<YT*>(y), channels,
                                                               (uint32_t)per_image, nvec);
        return launch_status("grn scale");
    };
    auto run_x = [&](auto yt) -> int {
        switch (x_dtype) {
            case VH_F32: return run(float{}, yt);
            case VH_BF16: return run(__nv_bfloat16{}, yt);
            default: return run(__half{}, yt);
        }
    };
    switch (y_dtype) {
        case VH_F32: return run_x(float{});
        case VH_BF16: return run_x(__nv_bfloat16{});
        default: return run_x(__half{});
    }
}

extern "C" int vh_layernorm_fwd(const void* x, int32_t x_dtype, const float* weight,
                                const float* bias, float eps, void* y, int32_t y_dtype, float* mean,
                                float* rstd, int64_t rows, int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!x || !weight || !bias || !y) return fail(VH_E_ARG, "vh_layernorm_fwd: null pointer argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(VH_E_DTYPE, "vh_layernorm_fwd: bad dtype");
    if (rows <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_layernorm_fwd: empty input");
    if (rows > ((int64_t)1 << 40)) return fail(VH_E_RANGE, "vh_layernorm_fwd: too many rows");
    const bool vec_ok = aligned(x, x_dtype == VH_F32 ? 16 : 8) && aligned(y, y_dtype == VH_F32 ? 16 : 8);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case VH_F32: return ln_run_y<float>(y_dtype, x, weight, bias, eps, y, mean, rstd, rows, channels, vec_ok, st);
        case VH_BF16: return ln_run_y<__nv_bfloat16>(y_dtype, x, weight, bias, eps, y, mean, rstd, rows, channels, vec_ok, st);
        default: return ln_run_y<__half>(y_dtype, x, weight, bias, eps, y, mean, rstd, rows, channels, vec_ok, st);
    }
}

extern "C" int vh_add_layernorm_fwd(const void* x, int32_t x_dtype, const void* r, int32_t r_dtype,
                                    void* sum_out, const float* weight, const float* bias, float eps, void* y,
                                    int32_t y_dtype, int64_t rows, int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!x || !r || !sum_out || !weight || !bias || !y)
        return fail(VH_E_ARG, "vh_add_layernorm_fwd: null pointer argument");
    if ((x_dtype != VH_F32 && x_dtype != VH_BF16) || (r_dtype != VH_F32 && r_dtype != VH_BF16) || !dtype_ok(y_dtype))
        return fail(VH_E_DTYPE, "vh_add_layernorm_fwd: x and r must be fp32 or bf16");
    if (rows <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_add_layernorm_fwd: empty input");
    if (channels % 8 || channels > 2048) return fail(VH_E_SHAPE, "vh_add_layernorm_fwd: channels must be a multiple of 8, at most 2048");
    if (rows > ((int64_t)1 << 40)) return fail(VH_E_RANGE, "vh_add_layernorm_fwd: too many rows");
    if (!aligned(x, 16) || !aligned(r, 16) || !aligned(sum_out, 16) || !aligned(y, 16) || !aligned(weight, 16) ||
        !aligned(bias, 16))
        return fail(VH_E_ALIGN, "vh_add_layernorm_fwd: pointers must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (x_dtype == VH_F32)
        return r_dtype == VH_F32 ? add_ln_y<float, float>(y_dtype, x, r, sum_out, weight, bias, eps, y, rows, channels, st)
                                 : add_ln_y<float, __nv_bfloat16>(y_dtype, x, r, sum_out, weight, bias, eps, y, rows, channels, st);
    return r_dtype == VH_F32 ? add_ln_y<__nv_bfloat16, float>(y_dtype, x, r, sum_out, weight, bias, eps, y, rows, channels, st)
                             : add_ln_y<__nv_bfloat16, __nv_bfloat16>(y_dtype, x, r, sum_out, weight, bias, eps, y, rows, channels, st);
}

// =========================== GRN without any device allocation ===========================
// Some callers cannot allocate device memory at the time they run GRN: inference servers and
// plugin hosts whose custom-op interface hands an op only its input and output buffers (no
// allocator, no workspace), and deployments that fix their device memory budget at start-up
// and forbid allocation afterwards (an allocation can fail, fragment the pool or, for
// cudaFree, synchronize the whole device).  vh_grn_fwd_noalloc serves them: it runs the same
// two GRN passes as vh_grn_fwd, but keeps the per-slice partial sums in a fixed array that is
// part of the library image on every device that loads it, so it allocates nothing.
namespace vh {
namespace {

// Partial sums [batch, splits, channels] fp32; 4 MiB per device, held until process exit.
constexpr int64_t kGrnNoAllocScratchFloats = int64_t(1) << 20;
static __device__ __align__(256) float g_grn_noalloc_scratch[kGrnNoAllocScratchFloats];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {nullptr};  // device address of the array, per device ordinal

// Device address of the scratch array on the current device (looked up once per device;
// in host code the array's name is only a host-side stand-in, never a device address).
int noalloc_scratch(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(VH_E_DEVICE, "vh_grn_fwd_noalloc: no usable current device");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_grn_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(VH_E_DEVICE, "vh_grn_fwd_noalloc: cudaGetSymbolAddress failed: %s",
                        cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}

}  // namespace
}  // namespace vh

extern "C" void vh_grn_noalloc_reset(void) {
    std::lock_guard<std::mutex> lock(vh::g_noalloc_mu);
    for (float*& p : vh::g_noalloc_ptr) p = nullptr;
}

extern "C" int vh_grn_fwd_noalloc(const void* x, int32_t x_dtype, const float* gamma,
                                  const float* beta, float eps, float* y, float* gx, float* inv_den,
                                  int32_t batch, int32_t height, int32_t width, int32_t channels,
                                  vh_stream_t stream) {
    clear_error();
    if (!x || !gamma || !beta || !y) return fail(VH_E_ARG, "vh_grn_fwd_noalloc: null pointer argument");
    if (!dtype_ok(x_dtype)) return fail(VH_E_DTYPE, "GRN supports FP32, FP16 and BF16 input");
    if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0)
        return fail(VH_E_SHAPE, "GRN expects nonempty input");
    if (channels % 4) return fail(VH_E_SHAPE, "vh_grn_fwd_noalloc: channels must be a multiple of 4");
    if (batch > 65535) return fail(VH_E_RANGE, "vh_grn_fwd_noalloc: batch must be <= 65535");
    if ((int64_t)batch * channels > kGrnNoAllocScratchFloats)
        return fail(VH_E_RANGE,
                    "vh_grn_fwd_noalloc: batch * channels = %lld exceeds the built-in scratch of %lld "
                    "values; use vh_grn_fwd with a caller-provided workspace",
                    (long long)batch * channels, (long long)kGrnNoAllocScratchFloats);
    if ((size_t)channels * 4 + 128 > 200 * 1024) return fail(VH_E_RANGE, "vh_grn_fwd_noalloc: too many channels");
    if (!aligned(x, x_dtype == VH_F32 ? 16 : 8) || !aligned(y, 16))
        return fail(VH_E_ALIGN, "vh_grn_fwd_noalloc: misaligned pointers");
    float* part = nullptr;
    const int rc = noalloc_scratch(&part);
    if (rc) return rc;
    const int64_t S = (int64_t)height * width;
    // Same two passes as vh_grn_fwd; the slice count shrinks when needed so that
    // batch * splits * channels partial sums fit the fixed array.
    int splits = grn_splits(batch, S);
    const int64_t fit = kGrnNoAllocScratchFloats / ((int64_t)batch * channels);
    if (splits > fit) splits = (int)fit;
    const int G = channels / 4;
    const int Geff = std::min(G, kGrnThreads);
    const int rph = kGrnThreads / Geff;
    const size_t red_bytes = sizeof(float) * (size_t)rph * Geff * 4;
    const size_t fac_bytes = sizeof(float) * ((size_t)channels + 32);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dim3 grid(splits, batch);
    auto run = [&](auto tag) -> int {
        using T = decltype(tag);
        const T* xp = static_cast<const T*>(x);
        if (!ensure_smem_attr(reinterpret_cast<const void*>(&grn_stats_kernel<T>), red_bytes) ||
            !ensure_smem_attr(reinterpret_cast<const void*>(&grn_apply_kernel<T>), fac_bytes))
            return fail(VH_E_DEVICE, "vh_grn_fwd_noalloc: shared memory");
        // Every partial sum is written (not accumulated) by the stats pass, so the array needs
        // no clearing between calls.
        grn_stats_kernel<T><<<grid, kGrnThreads, red_bytes, st>>>(xp, part, channels, S, splits);
        int r = launch_status("grn stats (no-alloc)");
        if (r) return r;
        grn_apply_kernel<T><<<grid, kGrnThreads, fac_bytes, st>>>(xp, part, gamma, beta, eps, y, gx,
                                                                   inv_den, channels, S, splits);
        return launch_status("grn apply (no-alloc)");
    };
    switch (x_dtype) {
        case VH_F32: return run(float{});
        case VH_BF16: return run(__nv_bfloat16{});
        default: return run(__half{});
    }
}
