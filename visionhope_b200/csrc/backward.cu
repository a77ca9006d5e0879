// Backward kernels of the HBM-bound operators on the path (training): query normalization,
// direction restoration + fusion, LayerNorm and GRN, with their C entry points.  Every
// reduction over pixels or rows runs in a fixed order (per-CTA partial sums, then one pass over
// the partials), so gradients are bit-reproducible from run to run.
#include <algorithm>
#include <climits>

#include "abi_util.h"
#include "common.cuh"

namespace vh {
namespace bwd {

constexpr int kThreads = 256;

// ---- query normalization (query_normalization.cu:78-134, 180-221) -------------------------
// q_out = q / max(||q||, 1e-12) per head vector.  d q = (g - q_out (q_out . g)) * inv, or
// g * inv where the norm was clamped (inv = 1e12).  One thread per vector, l fastest (the
// fp32 gradient rows are read contiguously); the result goes back to the [B, R, L, C] layout
// of q_raw in q_raw's dtype.
template <int D, typename T>
__global__ void __launch_bounds__(kThreads) qnorm_bwd_kernel(const float* __restrict__ g_out,
                                                             const float* __restrict__ q_out,
                                                             const float* __restrict__ inv_norm,
                                                             T* __restrict__ dq, int B, int R, int L,
                                                             int heads) {
    const int64_t n = (int64_t)B * R * heads * L;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    const int l = (int)(idx % L);
    const int64_t rest = idx / L;
    const int head = (int)(rest % heads);
    const int64_t br = rest / heads;
    float g[D], q[D];
#pragma unroll
    for (int i = 0; i < D; i += 4) {
        const float4 a = load4(g_out + idx * D + i), b = load4(q_out + idx * D + i);
        g[i] = a.x; g[i + 1] = a.y; g[i + 2] = a.z; g[i + 3] = a.w;
        q[i] = b.x; q[i + 1] = b.y; q[i + 2] = b.z; q[i + 3] = b.w;
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) dot = fmaf(g[i], q[i], dot);
    const float inv = inv_norm[(br * L + l) * heads + head];
    const bool clamped = inv > 9.999e11f;  // ||q|| < 1e-12: q_out = q * 1e12 is linear in q
    T* dst = dq + (br * L + l) * (int64_t)(heads * D) + (int64_t)head * D;
#pragma unroll
    for (int i = 0; i < D; i += 4) {
        float4 o;
        o.x = clamped ? g[i] * inv : (g[i] - q[i] * dot) * inv;
        o.y = clamped ? g[i + 1] * inv : (g[i + 1] - q[i + 1] * dot) * inv;
        o.z = clamped ? g[i + 2] * inv : (g[i + 2] - q[i + 2] * dot) * inv;
        o.w = clamped ? g[i + 3] * inv : (g[i + 3] - q[i + 3] * dot) * inv;
        store4(dst + i, o);
    }
}

template <typename T>
int qnorm_bwd_dispatch(int D, const float* g, const float* q, const float* inv, void* dq, int B, int R,
                       int L, int heads, cudaStream_t st) {
    const int64_t n = (int64_t)B * R * heads * L;
    const int grid = (int)((n + kThreads - 1) / kThreads);
    T* out = static_cast<T*>(dq);
    switch (D) {
        case 4: qnorm_bwd_kernel<4, T><<<grid, kThreads, 0, st>>>(g, q, inv, out, B, R, L, heads); break;
        case 8: qnorm_bwd_kernel<8, T><<<grid, kThreads, 0, st>>>(g, q, inv, out, B, R, L, heads); break;
        case 16: qnorm_bwd_kernel<16, T><<<grid, kThreads, 0, st>>>(g, q, inv, out, B, R, L, heads); break;
        case 32: qnorm_bwd_kernel<32, T><<<grid, kThreads, 0, st>>>(g, q, inv, out, B, R, L, heads); break;
        default: qnorm_bwd_kernel<64, T><<<grid, kThreads, 0, st>>>(g, q, inv, out, B, R, L, heads); break;
    }
    return launch_status("vh_qnorm_bwd");
}

// ---- direction restoration + fusion (direction_fusion.cu:123-502) -------------------------
// out[b, c, pix] = sum_d scale[d, c] (y_d + skip_d[c] x_d)[b, head, l_d(pix), i], c = head D + i,
// l_d the position of pixel pix in scan d.  So for every (b, d, pixel, c):
//   dy_d = scale[d, c] g,   dx_d = scale[d, c] skip_d[c] g,
//   dscale[d, c] += g (y_d + skip_d[c] x_d),   dskip_d[c] += g scale[d, c] x_d.
// CTA = (b, head, group of `tpc` tiles of 8 x 8 pixels): each tile's gradient is
// staged in shared memory first (read along whichever axis is contiguous), then each thread
// takes (pixel, group of 4 channels) items, always of the same channel group, and keeps its
// partial sums in registers across the CTA's tiles; the CTA adds them over its threads in a
// fixed order and writes one partial row per (image, tile group).  reduce_parts_kernel adds the
// partial rows in order.  The tile group depends on the sizes only, so the summation order is
// the same on every GPU.
constexpr int kPix = 64;  // an 8 x 8 pixel tile: rows of 8 pixels for the row scans and columns
                          // of 8 for the column scans, so every scan reads runs of 8 positions

__host__ __device__ inline int dirfuse_tiles(int H, int W) { return ((H + 7) / 8) * ((W + 7) / 8); }

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) dirfuse_bwd_kernel(
    const float* __restrict__ g, int64_t gsb, int64_t gsc, int64_t gsh, int64_t gsw, const T* __restrict__ y,
    const T* __restrict__ x, const float* __restrict__ skip, int skip_per_dir, const float* __restrict__ scale,
    T* __restrict__ dy, T* __restrict__ dx, float* __restrict__ part, int heads, int H, int W, int tpc) {
    constexpr int G4 = D / 4;
    static_assert(kThreads % G4 == 0, "a thread keeps one channel group");
    __shared__ float gt[D][kPix + 1];
    __shared__ float red[kThreads / G4][8][4];
    const int64_t L = (int64_t)H * W;
    const int C = heads * D;
    const int tiles = dirfuse_tiles(H, W);
    const int tcols = (W + 7) / 8;
    const int ngroups = (tiles + tpc - 1) / tpc;
    const int group = blockIdx.x % ngroups;
    const int head = (blockIdx.x / ngroups) % heads;
    const int b = blockIdx.x / (ngroups * heads);
    const bool pix_fast = gsc != 1;  // NCHW-like gradient: pixels contiguous per channel
    const int grp = threadIdx.x % G4;
    const int c0 = head * D + grp * 4;
    float sc[4][4], sk[4][4];
#pragma unroll
    for (int d = 0; d < 4; ++d)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            sc[d][e] = scale[d * C + c0 + e];
            sk[d][e] = skip[(skip_per_dir ? d * C : 0) + c0 + e];
        }
    float ps[4][4] = {}, pk[4][4] = {};
    const int tile_end = min(tiles, (group + 1) * tpc);
    for (int tile = group * tpc; tile < tile_end; ++tile) {
        const int ti0 = (tile / tcols) * 8, tj0 = (tile % tcols) * 8;
        __syncthreads();  // the previous tile's gradient has been read
        for (int it = threadIdx.x; it < D * kPix; it += kThreads) {
            const int k = pix_fast ? it % kPix : it / D, ch = pix_fast ? it / kPix : it % D;
            const int pi = ti0 + (k >> 3), pj = tj0 + (k & 7);
            float v = 0.f;
            if (pi < H && pj < W) v = g[b * gsb + (int64_t)(head * D + ch) * gsc + (int64_t)pi * gsh + (int64_t)pj * gsw];
            gt[ch][k] = v;
        }
        __syncthreads();
        for (int it = threadIdx.x; it < kPix * G4; it += kThreads) {
            const int k = it / G4;
            const int pi = ti0 + (k >> 3), pj = tj0 + (k & 7);
            if (pi >= H || pj >= W) continue;
            const int64_t lhw = (int64_t)pi * W + pj, lwh = (int64_t)pj * H + pi;
            const int64_t ls[4] = {lhw, L - 1 - lhw, lwh, L - 1 - lwh};
            const float gv[4] = {gt[grp * 4][k], gt[grp * 4 + 1][k], gt[grp * 4 + 2][k], gt[grp * 4 + 3][k]};
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int64_t off = ((((int64_t)b * 4 + d) * heads + head) * L + ls[d]) * D + grp * 4;
                const float4 yv = load4(y + off), xv = load4(x + off);
                const float yy[4] = {yv.x, yv.y, yv.z, yv.w}, xs[4] = {xv.x, xv.y, xv.z, xv.w};
                float o1[4], o2[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    o1[e] = sc[d][e] * gv[e];
                    o2[e] = sc[d][e] * sk[d][e] * gv[e];
                    ps[d][e] = fmaf(gv[e], fmaf(sk[d][e], xs[e], yy[e]), ps[d][e]);
                    pk[d][e] = fmaf(gv[e] * sc[d][e], xs[e], pk[d][e]);
                }
                store4(dy + off, make_float4(o1[0], o1[1], o1[2], o1[3]));
                store4(dx + off, make_float4(o2[0], o2[1], o2[2], o2[3]));
            }
        }
    }
    // Threads of one channel group: tid = grp + G4 * slot.  Stage, then add the slots in order.
    const int slot = threadIdx.x / G4;
    constexpr int kSlots = kThreads / G4;
    float* mine = &red[0][0][0];  // [slot][8][4] per group, in rounds of one group
    for (int gg = 0; gg < G4; ++gg) {
        if (grp == gg) {
#pragma unroll
            for (int d = 0; d < 4; ++d)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    mine[(slot * 8 + d) * 4 + e] = ps[d][e];
                    mine[(slot * 8 + 4 + d) * 4 + e] = pk[d][e];
                }
        }
        __syncthreads();
        if (threadIdx.x < 32) {  // 8 quantities x 4 channels of group gg
            const int q = threadIdx.x >> 2, e = threadIdx.x & 3;
            float sum = 0.f;
            for (int sl = 0; sl < kSlots; ++sl) sum += mine[(sl * 8 + q) * 4 + e];
            part[((int64_t)(b * ngroups + group) * 8 + q) * C + head * D + gg * 4 + e] = sum;
        }
        __syncthreads();
    }
}

// out[q][c] = sum_p part[p][q][c] for q < nq, partial rows p in order; CTA = (32 columns, q),
// threads (column, part lane), the part lanes added in lane order.
__global__ void __launch_bounds__(kThreads) reduce_parts_kernel(const float* __restrict__ part, int64_t nparts,
                                                                int nq, int C, float* __restrict__ out) {
    const int c = blockIdx.x * 32 + (threadIdx.x & 31);
    const int q = blockIdx.y;
    const int pl = threadIdx.x >> 5;
    constexpr int kL = kThreads / 32;  // part lanes
    float sum = 0.f;
    if (c < C) {
        // Eight loads in flight per batch; the adds stay in p order.
        int64_t p = pl;
        for (; p + 7 * kL < nparts; p += 8 * kL) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = part[((p + u * kL) * nq + q) * C + c];
#pragma unroll
            for (int u = 0; u < 8; ++u) sum += v[u];
        }
        for (; p < nparts; p += kL) sum += part[(p * nq + q) * C + c];
    }
    __shared__ float red[kThreads / 32][32];
    red[pl][threadIdx.x & 31] = sum;
    __syncthreads();
    if (pl == 0 && c < C) {
        float t = red[0][threadIdx.x];
        for (int k = 1; k < kThreads / 32; ++k) t += red[k][threadIdx.x];
        out[(int64_t)q * C + c] = t;
    }
}

int reduce_parts(const float* part, int64_t nparts, int nq, int C, float* out, cudaStream_t st) {
    reduce_parts_kernel<<<dim3((C + 31) / 32, nq), kThreads, 0, st>>>(part, nparts, nq, C, out);
    return launch_status("reduce of partial sums");
}

// dscale and dskip from the 8 summed rows: rows 0-3 dscale[d], rows 4-7 dskip[d]
// (added over d, in order, when the skip is shared).
__global__ void dirfuse_finish_kernel(const float* __restrict__ sums, int C, int skip_per_dir,
                                      float* __restrict__ dscale, float* __restrict__ dskip) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
#pragma unroll
    for (int d = 0; d < 4; ++d) dscale[d * C + c] = sums[d * C + c];
    if (skip_per_dir) {
#pragma unroll
        for (int d = 0; d < 4; ++d) dskip[d * C + c] = sums[(4 + d) * C + c];
    } else {
        dskip[c] = ((sums[4 * C + c] + sums[5 * C + c]) + sums[6 * C + c]) + sums[7 * C + c];
    }
}

// ---- LayerNorm over channels (layer_norm_cuda.py:59-119) ----------------------------------
// x_hat = (x - mean) rstd, y = w x_hat + b.  Per row r:
//   dx = rstd (w dy - mean_c(w dy) - x_hat mean_c(w dy x_hat)),
// and over rows: dw = sum_r dy x_hat, db = sum_r dy.
// ln_dx_kernel: eight lanes per row (two passes over the row: the sums, then dx).
// ln_param_kernel: CTA = (block of kLnRows rows, block of 32 channels), partial sums of
// the block written per CTA; reduce_parts_kernel adds them in row-block order.
constexpr int kLnRows = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads) ln_dx_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                         const float* __restrict__ w, const float* __restrict__ mean,
                                                         const float* __restrict__ rstd, T* __restrict__ dx,
                                                         int64_t rows, int C) {
    // Eight lanes per row, four rows per warp: each load instruction covers four 32-byte runs.
    const int lane = threadIdx.x & 31, sl = lane & 7;
    const int64_t r = ((int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * 4 + (lane >> 3);
    const bool live = r < rows;
    const float* g = dy + (live ? r : 0) * C;
    const T* xr = x + (live ? r : 0) * C;
    const float mu = live ? mean[r] : 0.f, rs = live ? rstd[r] : 0.f;
    float s1 = 0.f, s2 = 0.f;
    if (live)
        for (int c = sl; c < C; c += 8) {
            const float wg = w[c] * g[c];
            s1 += wg;
            s2 = fmaf(wg, (to_f(xr[c]) - mu) * rs, s2);
        }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (!live) return;
    const float invC = 1.f / (float)C;
    const float a = s1 * invC, bq = s2 * invC;
    T* dxr = dx + r * C;
    for (int c = sl; c < C; c += 8) {
        const float xh = (to_f(xr[c]) - mu) * rs;
        dxr[c] = from_f<T>((w[c] * g[c] - a - xh * bq) * rs);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) ln_param_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ rstd,
                                                            float* __restrict__ part, int64_t rows, int C) {
    const int c = blockIdx.y * 32 + (threadIdx.x & 31);
    const int rl = threadIdx.x >> 5;
    float sw = 0.f, sb = 0.f;
    if (c < C) {
        for (int k = rl; k < kLnRows; k += kThreads / 32) {
            const int64_t r = (int64_t)blockIdx.x * kLnRows + k;
            if (r >= rows) break;
            const float g = dy[r * C + c];
            sw = fmaf(g, (to_f(x[r * C + c]) - mean[r]) * rstd[r], sw);
            sb += g;
        }
    }
    __shared__ float red[kThreads / 32][2][32];
    red[rl][0][threadIdx.x & 31] = sw;
    red[rl][1][threadIdx.x & 31] = sb;
    __syncthreads();
    if (rl == 0 && c < C) {
        float a = red[0][0][threadIdx.x], bsum = red[0][1][threadIdx.x];
        for (int k = 1; k < kThreads / 32; ++k) {
            a += red[k][0][threadIdx.x];
            bsum += red[k][1][threadIdx.x];
        }
        part[((int64_t)blockIdx.x * 2) * C + c] = a;
        part[((int64_t)blockIdx.x * 2 + 1) * C + c] = bsum;
    }
}

// ln_fused_kernel (C <= kLnFusedMaxC): dx as ln_dx_kernel, with the parameter sums taken in
// the same pass.  Lane sl of a row owns channels sl + 8 m and keeps its dw, db sums over the
// CTA's rows in registers; the four row groups of a warp are added by shuffles, then the warps
// in order through shared memory, into one partial row per CTA of kLnRows rows.  dy and x are
// read from DRAM once (ln_param_kernel reads them a second time).
constexpr int kLnFusedMaxC = 128;

template <typename T, int NM>
__global__ void __launch_bounds__(kThreads) ln_fused_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ rstd, T* __restrict__ dx,
                                                            float* __restrict__ part, int64_t rows, int C) {
    const int lane = threadIdx.x & 31, sl = lane & 7, warp = threadIdx.x >> 5;
    float wv[NM], aw[NM], ab[NM];
#pragma unroll
    for (int m = 0; m < NM; ++m) {
        const int c = sl + 8 * m;
        wv[m] = c < C ? w[c] : 0.f;
        aw[m] = 0.f;
        ab[m] = 0.f;
    }
    const float invC = 1.f / (float)C;
    const int64_t r0 = (int64_t)blockIdx.x * kLnRows;
    for (int it = 0; it < kLnRows / 32; ++it) {  // the same trip count for every lane
        const int64_t r = r0 + it * 32 + warp * 4 + (lane >> 3);
        const bool live = r < rows;
        const float* gr = dy + (live ? r : 0) * C;
        const T* xr = x + (live ? r : 0) * C;
        const float mu = live ? mean[r] : 0.f, rs = live ? rstd[r] : 0.f;
        float gv[NM], xh[NM], s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const int c = sl + 8 * m;
            const bool ok = live && c < C;
            gv[m] = ok ? gr[c] : 0.f;
            xh[m] = ok ? (to_f(xr[c]) - mu) * rs : 0.f;
            const float wg = wv[m] * gv[m];
            s1 += wg;
            s2 = fmaf(wg, xh[m], s2);
            aw[m] = fmaf(gv[m], xh[m], aw[m]);
            ab[m] += gv[m];
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (live) {
            const float a = s1 * invC, bq = s2 * invC;
            T* dxr = dx + r * C;
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                const int c = sl + 8 * m;
                if (c < C) dxr[c] = from_f<T>((wv[m] * gv[m] - a - xh[m] * bq) * rs);
            }
        }
    }
    __shared__ float red[kThreads / 32][2][kLnFusedMaxC];
#pragma unroll
    for (int m = 0; m < NM; ++m) {
        aw[m] += __shfl_xor_sync(0xffffffffu, aw[m], 8);
        ab[m] += __shfl_xor_sync(0xffffffffu, ab[m], 8);
        aw[m] += __shfl_xor_sync(0xffffffffu, aw[m], 16);
        ab[m] += __shfl_xor_sync(0xffffffffu, ab[m], 16);
    }
    if (lane < 8) {
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const int c = sl + 8 * m;
            if (c < C) {
                red[warp][0][c] = aw[m];
                red[warp][1][c] = ab[m];
            }
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * C; e += kThreads) {
        const int q = e / C, c = e - q * C;
        float t = red[0][q][c];
        for (int k = 1; k < kThreads / 32; ++k) t += red[k][q][c];
        part[((int64_t)blockIdx.x * 2 + q) * C + c] = t;
    }
}

// ln_fused_wide_kernel (kLnFusedMaxC < C <= kLnWideMaxC): the one-pass backward with a warp
// per row, lane l owning channels l + 32 m; the same block of kLnRows rows per CTA (32 rows per
// warp), the warps' dw, db sums added in order through shared memory.
constexpr int kLnWideMaxC = 512;

template <typename T, int NM>
__global__ void __launch_bounds__(kThreads) ln_fused_wide_kernel(const float* __restrict__ dy,
                                                                 const T* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ mean,
                                                                 const float* __restrict__ rstd,
                                                                 T* __restrict__ dx, float* __restrict__ part,
                                                                 int64_t rows, int C) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float wv[NM], aw[NM], ab[NM];
#pragma unroll
    for (int m = 0; m < NM; ++m) {
        const int c = lane + 32 * m;
        wv[m] = c < C ? w[c] : 0.f;
        aw[m] = 0.f;
        ab[m] = 0.f;
    }
    const float invC = 1.f / (float)C;
    const int64_t r0 = (int64_t)blockIdx.x * kLnRows;
    for (int it = 0; it < kLnRows / (kThreads / 32); ++it) {
        const int64_t r = r0 + it * (kThreads / 32) + warp;
        if (r >= rows) break;  // uniform across the warp
        const float* gr = dy + r * C;
        const T* xr = x + r * C;
        const float mu = mean[r], rs = rstd[r];
        float gv[NM], xh[NM], s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const int c = lane + 32 * m;
            const bool ok = c < C;
            gv[m] = ok ? gr[c] : 0.f;
            xh[m] = ok ? (to_f(xr[c]) - mu) * rs : 0.f;
            const float wg = wv[m] * gv[m];
            s1 += wg;
            s2 = fmaf(wg, xh[m], s2);
            aw[m] = fmaf(gv[m], xh[m], aw[m]);
            ab[m] += gv[m];
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        const float a = s1 * invC, bq = s2 * invC;
        T* dxr = dx + r * C;
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const int c = lane + 32 * m;
            if (c < C) dxr[c] = from_f<T>((wv[m] * gv[m] - a - xh[m] * bq) * rs);
        }
    }
    __shared__ float red[kThreads / 32][2][kLnWideMaxC];
#pragma unroll
    for (int m = 0; m < NM; ++m) {
        const int c = lane + 32 * m;
        if (c < C) {
            red[warp][0][c] = aw[m];
            red[warp][1][c] = ab[m];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * C; e += kThreads) {
        const int q = e / C, c = e - q * C;
        float t = red[0][q][c];
        for (int k = 1; k < kThreads / 32; ++k) t += red[k][q][c];
        part[((int64_t)blockIdx.x * 2 + q) * C + c] = t;
    }
}

// ---- GRN (grn_cuda.cu:126-265) ------------------------------------------------------------
// y = x (1 + gamma Nx) + beta, Nx = Gx inv, Gx[b, c] = ||x[b, :, c]||, inv = 1 / (mean_c Gx + eps).
// With t[b, c] = sum_s dy x and s = gamma t:
//   dgamma = sum_b Nx t,  dbeta = sum_b sum_s dy,
//   dGx = s inv - (sum_c s Gx) inv^2 / C,
//   dx = dy (1 + gamma Nx) + dGx x / Gx   (0 where Gx = 0).
// grn_stats_bwd_kernel: CTA = (b, block of 32 channels, slice of the pixels), pixel lanes
// reduced in lane order; the slices' partial sums are added in slice order afterwards.
template <typename T>
__global__ void __launch_bounds__(kThreads) grn_stats_bwd_kernel(const float* __restrict__ dy,
                                                                 const T* __restrict__ x, int S, int C, int nsl,
                                                                 float* __restrict__ t_part,
                                                                 float* __restrict__ db_part) {
    const int b = blockIdx.x;
    const int c = blockIdx.y * 32 + (threadIdx.x & 31);
    const int sl = blockIdx.z;
    const int pl = threadIdx.x >> 5;
    const int per = (S + nsl - 1) / nsl;
    const int s0 = sl * per, s1 = min(S, s0 + per);
    float t = 0.f, sb = 0.f;
    if (c < C) {
        const int64_t base = (int64_t)b * S * C + c;
        for (int s = s0 + pl; s < s1; s += kThreads / 32) {
            const float g = dy[base + (int64_t)s * C];
            t = fmaf(g, to_f(x[base + (int64_t)s * C]), t);
            sb += g;
        }
    }
    __shared__ float red[kThreads / 32][2][32];
    red[pl][0][threadIdx.x & 31] = t;
    red[pl][1][threadIdx.x & 31] = sb;
    __syncthreads();
    if (pl == 0 && c < C) {
        float a = red[0][0][threadIdx.x], bsum = red[0][1][threadIdx.x];
        for (int k = 1; k < kThreads / 32; ++k) {
            a += red[k][0][threadIdx.x];
            bsum += red[k][1][threadIdx.x];
        }
        t_part[((int64_t)b * nsl + sl) * C + c] = a;
        db_part[((int64_t)b * nsl + sl) * C + c] = bsum;
    }
}

// t[b, c] and dbeta_bc[b, c]: the slices added in order.
__global__ void grn_slices_kernel(const float* __restrict__ t_part, const float* __restrict__ db_part, int B, int C,
                                  int nsl, float* __restrict__ t, float* __restrict__ dbeta_bc) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * C) return;
    const int64_t b = i / C, c = i % C;
    float a = 0.f, bsum = 0.f;
    for (int sl = 0; sl < nsl; ++sl) {
        a += t_part[(b * nsl + sl) * C + c];
        bsum += db_part[(b * nsl + sl) * C + c];
    }
    t[i] = a;
    dbeta_bc[i] = bsum;
}

// One CTA per image: the factors of dx = dy f1 + x f2 for each channel, f1 = 1 + gamma Nx and
// f2 = dGx / Gx (0 where Gx = 0), with dGx = gamma t inv - (sum_c gamma t Gx) inv^2 / C (the sum
// over channels in a fixed tree order).
__global__ void __launch_bounds__(kThreads) grn_factor_bwd_kernel(const float* __restrict__ t,
                                                                  const float* __restrict__ gamma,
                                                                  const float* __restrict__ gx,
                                                                  const float* __restrict__ inv_den, int C,
                                                                  float* __restrict__ f1, float* __restrict__ f2) {
    const int b = blockIdx.x;
    __shared__ float red[kThreads / 32];
    float sum = 0.f;
    for (int c = threadIdx.x; c < C; c += kThreads) sum = fmaf(gamma[c] * t[(int64_t)b * C + c], gx[(int64_t)b * C + c], sum);
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kThreads / 32; ++k) tot += red[k];
    const float inv = inv_den[b];
    for (int c = threadIdx.x; c < C; c += kThreads) {
        const int64_t i = (int64_t)b * C + c;
        const float g = gx[i];
        const float dgx = gamma[c] * t[i] * inv - tot * inv * inv / (float)C;
        f1[i] = fmaf(gamma[c], g * inv, 1.f);
        f2[i] = g > 0.f ? dgx / g : 0.f;
    }
}

// dx = dy f1[b, c] + x f2[b, c]; grid (vector blocks, image).  Vectors of 4 channels when C is a
// multiple of 4 (VEC), single elements otherwise.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) grn_dx_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                          const float* __restrict__ f1, const float* __restrict__ f2,
                                                          T* __restrict__ dx, int S, int C) {
    const int b = blockIdx.y;
    const int W = VEC ? 4 : 1;
    const int64_t per = (int64_t)S * C / W;
    const int64_t base = (int64_t)b * S * C;
    const float* f1b = f1 + (int64_t)b * C;
    const float* f2b = f2 + (int64_t)b * C;
    // The channel of vector v, v mod (C / W), kept up to date by adding the stride's remainder
    // (no 64-bit division per vector).
    const int CV = C / W;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    const int smod = (int)(stride % CV);
    int64_t v = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    int cv = (int)(v % CV);
    for (; v < per; v += stride, cv = cv + smod >= CV ? cv + smod - CV : cv + smod) {
        const int64_t i = base + v * W;
        const int c = cv * W;
        if constexpr (VEC) {
            const float4 g = load4(dy + i), xv = load4(x + i), a = load4(f1b + c), bq = load4(f2b + c);
            store4(dx + i, make_float4(fmaf(g.x, a.x, xv.x * bq.x), fmaf(g.y, a.y, xv.y * bq.y),
                                       fmaf(g.z, a.z, xv.z * bq.z), fmaf(g.w, a.w, xv.w * bq.w)));
        } else {
            dx[i] = from_f<T>(fmaf(dy[i], f1b[c], to_f(x[i]) * f2b[c]));
        }
    }
}

// dgamma[c] = sum_b Nx[b, c] t[b, c], dbeta[c] = sum_b dbeta_bc[b, c], b in order.
__global__ void __launch_bounds__(kThreads) grn_param_kernel(const float* __restrict__ t, const float* __restrict__ gx,
                                                             const float* __restrict__ inv_den,
                                                             const float* __restrict__ dbeta_bc, int B, int C,
                                                             float* __restrict__ dgamma, float* __restrict__ dbeta) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float a = 0.f, bsum = 0.f;
    int b = 0;
    // Eight images' loads in flight per batch; the sums stay in image order.
    for (; b + 8 <= B; b += 8) {
        float g[8], iv[8], tv[8], db[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int64_t i = (int64_t)(b + u) * C + c;
            g[u] = gx[i];
            iv[u] = inv_den[b + u];
            tv[u] = t[i];
            db[u] = dbeta_bc[i];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            a = fmaf(g[u] * iv[u], tv[u], a);
            bsum += db[u];
        }
    }
    for (; b < B; ++b) {
        a = fmaf(gx[(int64_t)b * C + c] * inv_den[b], t[(int64_t)b * C + c], a);
        bsum += dbeta_bc[(int64_t)b * C + c];
    }
    dgamma[c] = a;
    dbeta[c] = bsum;
}

}  // namespace bwd
}  // namespace vh

using namespace vh;
using namespace vh::bwd;

namespace {

template <typename F>
int by_dtype(int dt, F&& f) {
    switch (dt) {
        case VH_F32: return f(float{});
        case VH_BF16: return f(__nv_bfloat16{});
        default: return f(__half{});
    }
}

// Tiles per CTA of the direction-fusion backward: about 2368 CTAs (two waves of eight per SM
// on 148 SMs), at most 16 tiles; from the sizes alone.
int dirfuse_tpc(int batch, int heads, int height, int width) {
    const int64_t tiles = dirfuse_tiles(height, width);
    const int64_t want = ((int64_t)batch * heads * tiles + 2367) / 2368;
    return (int)std::max<int64_t>(1, std::min<int64_t>(16, want));
}

int64_t dirfuse_parts(int batch, int heads, int height, int width) {
    const int64_t tiles = dirfuse_tiles(height, width);
    const int tpc = dirfuse_tpc(batch, heads, height, width);
    return (int64_t)batch * ((tiles + tpc - 1) / tpc);
}

}  // namespace

extern "C" int vh_qnorm_bwd(const float* grad_out, const float* q_out, const float* inv_norm, void* grad_q,
                            int32_t q_dtype, int32_t batch, int32_t dirs, int32_t length, int32_t heads,
                            int32_t head_dim, vh_stream_t stream) {
    clear_error();
    if (!grad_out || !q_out || !inv_norm || !grad_q) return fail(VH_E_ARG, "vh_qnorm_bwd: null pointer argument");
    if (!dtype_ok(q_dtype)) return fail(VH_E_DTYPE, "vh_qnorm_bwd: bad dtype");
    if (!head_dim_ok(head_dim)) return fail(VH_E_HEADDIM, "Unsupported qnorm head dimension %d", head_dim);
    if (batch <= 0 || dirs <= 0 || length <= 0 || heads <= 0)
        return fail(VH_E_SHAPE, "vh_qnorm_bwd: sizes must be positive");
    if (!aligned(grad_out, 16) || !aligned(q_out, 16) || !aligned(grad_q, q_dtype == VH_F32 ? 16 : 8))
        return fail(VH_E_ALIGN, "vh_qnorm_bwd: misaligned pointers");
    if ((int64_t)batch * dirs * heads * length > ((int64_t)1 << 40))
        return fail(VH_E_RANGE, "vh_qnorm_bwd: too many vectors");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return by_dtype(q_dtype, [&](auto t) {
        using T = decltype(t);
        return qnorm_bwd_dispatch<T>(head_dim, grad_out, q_out, inv_norm, grad_q, batch, dirs, length, heads, st);
    });
}

extern "C" int64_t vh_dirfuse_bwd_workspace_bytes(int32_t batch, int32_t heads, int32_t height, int32_t width,
                                                  int32_t head_dim) {
    if (batch <= 0 || heads <= 0 || height <= 0 || width <= 0 || head_dim <= 0) return 0;
    return (dirfuse_parts(batch, heads, height, width) + 1) * 8 * (int64_t)heads * head_dim * (int64_t)sizeof(float);
}

extern "C" int vh_dirfuse_bwd(const float* grad_out, int64_t gs_b, int64_t gs_c, int64_t gs_h, int64_t gs_w,
                              const void* y, const void* x, int32_t io_dtype, const float* skip,
                              int32_t skip_per_dir, const float* scale, void* grad_y, void* grad_x,
                              float* grad_skip, float* grad_scale, void* workspace, int64_t workspace_bytes,
                              int32_t batch, int32_t heads, int32_t height, int32_t width, int32_t head_dim,
                              vh_stream_t stream) {
    clear_error();
    if (!grad_out || !y || !x || !skip || !scale || !grad_y || !grad_x || !grad_skip || !grad_scale || !workspace)
        return fail(VH_E_ARG, "vh_dirfuse_bwd: null pointer argument");
    if (!dtype_ok(io_dtype)) return fail(VH_E_DTYPE, "vh_dirfuse_bwd: bad dtype");
    if (batch <= 0 || heads <= 0 || height <= 0 || width <= 0 || head_dim <= 0)
        return fail(VH_E_SHAPE, "vh_dirfuse_bwd: sizes must be positive");
    if (workspace_bytes < vh_dirfuse_bwd_workspace_bytes(batch, heads, height, width, head_dim))
        return fail(VH_E_ARG, "vh_dirfuse_bwd: workspace too small");
    const int64_t L = (int64_t)height * width;
    if ((int64_t)batch * 4 * L * heads * head_dim > ((int64_t)1 << 40) || batch > 65535)
        return fail(VH_E_RANGE, "vh_dirfuse_bwd: too many elements");
    const int C = heads * head_dim;
    const int tiles = dirfuse_tiles(height, width);
    if (!head_dim_ok(head_dim)) return fail(VH_E_HEADDIM, "vh_dirfuse_bwd: unsupported head_dim %d", head_dim);
    if (!aligned(y, io_dtype == VH_F32 ? 16 : 8) || !aligned(x, io_dtype == VH_F32 ? 16 : 8) ||
        !aligned(grad_y, io_dtype == VH_F32 ? 16 : 8) || !aligned(grad_x, io_dtype == VH_F32 ? 16 : 8))
        return fail(VH_E_ALIGN, "vh_dirfuse_bwd: misaligned pointers");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int tpc = dirfuse_tpc(batch, heads, height, width);
    const int64_t nparts = dirfuse_parts(batch, heads, height, width);
    float* part = static_cast<float*>(workspace);
    float* sums = part + nparts * 8 * C;
    const int64_t grid = (int64_t)batch * heads * ((tiles + tpc - 1) / tpc);
    if (grid > INT32_MAX) return fail(VH_E_RANGE, "vh_dirfuse_bwd: too many tiles");
    int rc = by_dtype(io_dtype, [&](auto t) {
        using T = decltype(t);
        const T* yp = static_cast<const T*>(y);
        const T* xp = static_cast<const T*>(x);
        T* dyp = static_cast<T*>(grad_y);
        T* dxp = static_cast<T*>(grad_x);
        const int spd = skip_per_dir ? 1 : 0;
        switch (head_dim) {
            case 4: dirfuse_bwd_kernel<4, T><<<(unsigned)grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, yp, xp, skip, spd, scale, dyp, dxp, part, heads, height, width, tpc); break;
            case 8: dirfuse_bwd_kernel<8, T><<<(unsigned)grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, yp, xp, skip, spd, scale, dyp, dxp, part, heads, height, width, tpc); break;
            case 16: dirfuse_bwd_kernel<16, T><<<(unsigned)grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, yp, xp, skip, spd, scale, dyp, dxp, part, heads, height, width, tpc); break;
            case 32: dirfuse_bwd_kernel<32, T><<<(unsigned)grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, yp, xp, skip, spd, scale, dyp, dxp, part, heads, height, width, tpc); break;
            default: dirfuse_bwd_kernel<64, T><<<(unsigned)grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, yp, xp, skip, spd, scale, dyp, dxp, part, heads, height, width, tpc); break;
        }
        return launch_status("vh_dirfuse_bwd");
    });
    if (rc) return rc;
    reduce_parts_kernel<<<dim3((C + 31) / 32, 8), kThreads, 0, st>>>(part, nparts, 8, C, sums);
    if ((rc = launch_status("vh_dirfuse_bwd (reduce)"))) return rc;
    dirfuse_finish_kernel<<<(C + kThreads - 1) / kThreads, kThreads, 0, st>>>(sums, C, skip_per_dir ? 1 : 0,
                                                                              grad_scale, grad_skip);
    return launch_status("vh_dirfuse_bwd (finish)");
}

extern "C" int64_t vh_layernorm_bwd_workspace_bytes(int64_t rows, int32_t channels) {
    if (rows <= 0 || channels <= 0) return 0;
    return (((rows + kLnRows - 1) / kLnRows) + 1) * 2 * (int64_t)channels * (int64_t)sizeof(float);
}

extern "C" int vh_layernorm_bwd(const float* grad_y, const void* x, int32_t x_dtype, const float* weight,
                                const float* mean, const float* rstd, void* grad_x, float* grad_weight,
                                float* grad_bias, void* workspace, int64_t workspace_bytes, int64_t rows,
                                int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!grad_y || !x || !weight || !mean || !rstd || !grad_x || !grad_weight || !grad_bias || !workspace)
        return fail(VH_E_ARG, "vh_layernorm_bwd: null pointer argument");
    if (!dtype_ok(x_dtype)) return fail(VH_E_DTYPE, "vh_layernorm_bwd: bad dtype");
    if (rows <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_layernorm_bwd: sizes must be positive");
    if (workspace_bytes < vh_layernorm_bwd_workspace_bytes(rows, channels))
        return fail(VH_E_ARG, "vh_layernorm_bwd: workspace too small");
    const int64_t rblocks = (rows + kLnRows - 1) / kLnRows;
    if (rows * channels > ((int64_t)1 << 40) || rblocks > INT32_MAX || (channels + 31) / 32 > 65535)
        return fail(VH_E_RANGE, "vh_layernorm_bwd: too many elements");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    int rc = by_dtype(x_dtype, [&](auto t) {
        using T = decltype(t);
        if (channels <= kLnFusedMaxC) {
            if (channels <= 64)
                ln_fused_kernel<T, 8><<<(unsigned)rblocks, kThreads, 0, st>>>(
                    grad_y, static_cast<const T*>(x), weight, mean, rstd, static_cast<T*>(grad_x), part, rows, channels);
            else
                ln_fused_kernel<T, 16><<<(unsigned)rblocks, kThreads, 0, st>>>(
                    grad_y, static_cast<const T*>(x), weight, mean, rstd, static_cast<T*>(grad_x), part, rows, channels);
            return launch_status("vh_layernorm_bwd (fused)");
        }
        if (channels <= kLnWideMaxC) {
            if (channels <= 256)
                ln_fused_wide_kernel<T, 8><<<(unsigned)rblocks, kThreads, 0, st>>>(
                    grad_y, static_cast<const T*>(x), weight, mean, rstd, static_cast<T*>(grad_x), part, rows, channels);
            else
                ln_fused_wide_kernel<T, 16><<<(unsigned)rblocks, kThreads, 0, st>>>(
                    grad_y, static_cast<const T*>(x), weight, mean, rstd, static_cast<T*>(grad_x), part, rows, channels);
            return launch_status("vh_layernorm_bwd (fused, wide rows)");
        }
        const int64_t grid = (rows + 4 * (kThreads / 32) - 1) / (4 * (kThreads / 32));
        if (grid > INT32_MAX) return fail(VH_E_RANGE, "vh_layernorm_bwd: too many rows");
        ln_dx_kernel<T><<<(unsigned)grid, kThreads, 0, st>>>(grad_y, static_cast<const T*>(x), weight, mean, rstd,
                                                              static_cast<T*>(grad_x), rows, channels);
        int r = launch_status("vh_layernorm_bwd (dx)");
        if (r) return r;
        ln_param_kernel<T><<<dim3((unsigned)rblocks, (channels + 31) / 32), kThreads, 0, st>>>(
            grad_y, static_cast<const T*>(x), mean, rstd, part, rows, channels);
        return launch_status("vh_layernorm_bwd (params)");
    });
    if (rc) return rc;
    float* sums = part + rblocks * 2 * channels;
    reduce_parts_kernel<<<dim3((channels + 31) / 32, 2), kThreads, 0, st>>>(part, rblocks, 2, channels, sums);
    if ((rc = launch_status("vh_layernorm_bwd (reduce)"))) return rc;
    if (cudaMemcpyAsync(grad_weight, sums, sizeof(float) * channels, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(grad_bias, sums + channels, sizeof(float) * channels, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return fail(VH_E_DEVICE, "vh_layernorm_bwd: copy of the parameter gradients failed");
    return 0;
}

namespace {
constexpr int kGrnMaxSlices = 16;
// Pixel slices per image: enough CTAs for about four per SM.
int grn_slices(int batch, int channels, int64_t S) {
    const int64_t ctas = (int64_t)batch * ((channels + 31) / 32);
    int64_t n = (4 * (int64_t)sm_count() + ctas - 1) / ctas;
    n = std::min<int64_t>(n, std::max<int64_t>(1, S / 64));
    return (int)std::max<int64_t>(1, std::min<int64_t>(n, kGrnMaxSlices));
}
}  // namespace

extern "C" int64_t vh_grn_bwd_workspace_bytes(int32_t batch, int32_t channels) {
    if (batch <= 0 || channels <= 0) return 0;
    return (4 + 2 * kGrnMaxSlices) * (int64_t)batch * channels * (int64_t)sizeof(float);
}

extern "C" int vh_grn_bwd(const float* grad_y, const void* x, int32_t x_dtype, const float* gamma, const float* gx,
                          const float* inv_den, void* grad_x, float* grad_gamma, float* grad_beta, void* workspace,
                          int64_t workspace_bytes, int32_t batch, int32_t height, int32_t width, int32_t channels,
                          vh_stream_t stream) {
    clear_error();
    if (!grad_y || !x || !gamma || !gx || !inv_den || !grad_x || !grad_gamma || !grad_beta || !workspace)
        return fail(VH_E_ARG, "vh_grn_bwd: null pointer argument");
    if (!dtype_ok(x_dtype)) return fail(VH_E_DTYPE, "vh_grn_bwd: bad dtype");
    if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0)
        return fail(VH_E_SHAPE, "vh_grn_bwd: sizes must be positive");
    if (workspace_bytes < vh_grn_bwd_workspace_bytes(batch, channels))
        return fail(VH_E_ARG, "vh_grn_bwd: workspace too small");
    const int64_t S = (int64_t)height * width;
    const int64_t n = (int64_t)batch * S * channels;
    if (n > ((int64_t)1 << 40) || S > INT32_MAX || (channels + 31) / 32 > 65535)
        return fail(VH_E_RANGE, "vh_grn_bwd: too many elements");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* t = static_cast<float*>(workspace);
    float* dbeta_bc = t + (int64_t)batch * channels;
    float* f1 = dbeta_bc + (int64_t)batch * channels;
    float* f2 = f1 + (int64_t)batch * channels;
    float* t_part = f2 + (int64_t)batch * channels;
    const int nsl = grn_slices(batch, channels, S);
    float* db_part = t_part + (int64_t)batch * nsl * channels;
    if (batch > 65535) return fail(VH_E_RANGE, "vh_grn_bwd: batch above 65535");
    return by_dtype(x_dtype, [&](auto tag) {
        using T = decltype(tag);
        const T* xp = static_cast<const T*>(x);
        grn_stats_bwd_kernel<T><<<dim3(batch, (channels + 31) / 32, nsl), kThreads, 0, st>>>(
            grad_y, xp, (int)S, channels, nsl, t_part, db_part);
        int r = launch_status("vh_grn_bwd (stats)");
        if (r) return r;
        const int64_t bc = (int64_t)batch * channels;
        grn_slices_kernel<<<(unsigned)((bc + kThreads - 1) / kThreads), kThreads, 0, st>>>(t_part, db_part, batch,
                                                                                           channels, nsl, t, dbeta_bc);
        if ((r = launch_status("vh_grn_bwd (slices)"))) return r;
        grn_factor_bwd_kernel<<<batch, kThreads, 0, st>>>(t, gamma, gx, inv_den, channels, f1, f2);
        if ((r = launch_status("vh_grn_bwd (factors)"))) return r;
        const bool vec = channels % 4 == 0 && aligned(grad_y, 16) && aligned(x, 4 * dtype_size(x_dtype)) &&
                         aligned(grad_x, 4 * dtype_size(x_dtype));
        const int64_t per = S * channels / (vec ? 4 : 1);
        const unsigned gx_blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((per + kThreads - 1) / kThreads,
                                                                                     (int64_t)sm_count() * 8 / batch + 1));
        if (vec)
            grn_dx_kernel<T, true><<<dim3(gx_blocks, batch), kThreads, 0, st>>>(grad_y, xp, f1, f2, static_cast<T*>(grad_x),
                                                                               (int)S, channels);
        else
            grn_dx_kernel<T, false><<<dim3(gx_blocks, batch), kThreads, 0, st>>>(grad_y, xp, f1, f2, static_cast<T*>(grad_x),
                                                                                (int)S, channels);
        if ((r = launch_status("vh_grn_bwd (dx)"))) return r;
        grn_param_kernel<<<(channels + 63) / 64, 64, 0, st>>>(t, gx, inv_den, dbeta_bc, batch, channels, grad_gamma,
                                                             grad_beta);
        return launch_status("vh_grn_bwd (params)");
    });
}
