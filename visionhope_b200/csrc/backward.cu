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
// CTA = (b, tile of kPix pixels, block of 32 channels); thread (channel lane, pixel lane).
// Each CTA writes its per-channel partial sums; dirfuse_reduce_kernel adds the partials of
// all CTAs in index order.
constexpr int kPix = 64;
constexpr int kPixLanes = kThreads / 32;

__device__ __forceinline__ int64_t scan_pos(int d, int64_t pix, int H, int W) {
    const int64_t L = (int64_t)H * W;
    const int64_t i = pix / W, j = pix - i * W;
    switch (d) {
        case 0: return pix;
        case 1: return L - 1 - pix;
        case 2: return j * H + i;
        default: return L - 1 - (j * H + i);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dirfuse_bwd_kernel(
    const float* __restrict__ g, int64_t gsb, int64_t gsc, int64_t gsh, int64_t gsw, const T* __restrict__ y,
    const T* __restrict__ x, const float* __restrict__ skip, int skip_per_dir, const float* __restrict__ scale,
    T* __restrict__ dy, T* __restrict__ dx, float* __restrict__ part, int heads, int H, int W, int D) {
    const int C = heads * D;
    const int64_t L = (int64_t)H * W;
    const int tiles = (int)((L + kPix - 1) / kPix);
    const int b = blockIdx.z;
    const int tile = blockIdx.x;
    const int c = blockIdx.y * 32 + (threadIdx.x & 31);
    const int pl = threadIdx.x >> 5;
    float ps[4] = {0.f, 0.f, 0.f, 0.f}, pk[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < C) {
        const int head = c / D, i = c - head * D;
        float sc[4], sk[4];
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            sc[d] = scale[d * C + c];
            sk[d] = skip[(skip_per_dir ? d * C : 0) + c];
        }
        for (int k = pl; k < kPix; k += kPixLanes) {
            const int64_t pix = (int64_t)tile * kPix + k;
            if (pix >= L) break;
            const int64_t pi = pix / W, pj = pix - pi * W;
            const float gv = g[b * gsb + c * gsc + pi * gsh + pj * gsw];
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int64_t o = (((int64_t)b * 4 + d) * heads + head) * L * D + scan_pos(d, pix, H, W) * D + i;
                const float yv = to_f(y[o]), xv = to_f(x[o]);
                dy[o] = from_f<T>(sc[d] * gv);
                dx[o] = from_f<T>(sc[d] * sk[d] * gv);
                ps[d] = fmaf(gv, fmaf(sk[d], xv, yv), ps[d]);
                pk[d] = fmaf(gv * sc[d], xv, pk[d]);
            }
        }
    }
    // Reduce over the pixel lanes in lane order, then write this CTA's partials.
    __shared__ float red[kPixLanes][8][32];
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        red[pl][d][threadIdx.x & 31] = ps[d];
        red[pl][4 + d][threadIdx.x & 31] = pk[d];
    }
    __syncthreads();
    if (pl == 0 && c < C) {
        float s[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) s[q] = red[0][q][threadIdx.x];
        for (int r = 1; r < kPixLanes; ++r)
#pragma unroll
            for (int q = 0; q < 8; ++q) s[q] += red[r][q][threadIdx.x];
        const int64_t cta = (int64_t)b * tiles + tile;
        float* dst = part + cta * 8 * C;
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q * C + c] = s[q];
    }
}

// dscale[d, c] and dskip (C or 4 C values) from the partials of `nparts` CTAs, in CTA order.
__global__ void __launch_bounds__(kThreads) dirfuse_reduce_kernel(const float* __restrict__ part, int64_t nparts,
                                                                  int C, int skip_per_dir, float* __restrict__ dscale,
                                                                  float* __restrict__ dskip) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int64_t p = 0; p < nparts; ++p)
#pragma unroll
        for (int q = 0; q < 8; ++q) s[q] += part[p * 8 * C + q * C + c];
#pragma unroll
    for (int d = 0; d < 4; ++d) dscale[d * C + c] = s[d];
    if (skip_per_dir) {
#pragma unroll
        for (int d = 0; d < 4; ++d) dskip[d * C + c] = s[4 + d];
    } else {
        dskip[c] = ((s[4] + s[5]) + s[6]) + s[7];
    }
}


// ---- LayerNorm over channels (layer_norm_cuda.py:59-119) ----------------------------------
// x_hat = (x - mean) rstd, y = w x_hat + b.  Per row r:
//   dx = rstd (w dy - mean_c(w dy) - x_hat mean_c(w dy x_hat)),
// and over rows: dw = sum_r dy x_hat, db = sum_r dy.
// ln_dx_kernel: one warp per row, lanes over channels (two passes over the row: the sums, then
// dx).  ln_param_kernel: CTA = (block of kLnRows rows, block of 32 channels), partial sums of
// the block written per CTA; param_reduce_kernel adds them in row-block order.
constexpr int kLnRows = 64;

template <typename T>
__global__ void __launch_bounds__(kThreads) ln_dx_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                         const float* __restrict__ w, const float* __restrict__ mean,
                                                         const float* __restrict__ rstd, T* __restrict__ dx,
                                                         int64_t rows, int C) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const float* g = dy + r * C;
    const T* xr = x + r * C;
    const float mu = mean[r], rs = rstd[r];
    float s1 = 0.f, s2 = 0.f;
    for (int c = lane; c < C; c += 32) {
        const float wg = w[c] * g[c];
        s1 += wg;
        s2 = fmaf(wg, (to_f(xr[c]) - mu) * rs, s2);
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float invC = 1.f / (float)C;
    const float a = s1 * invC, bq = s2 * invC;
    T* dxr = dx + r * C;
    for (int c = lane; c < C; c += 32) {
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

// out0[c] = sum_p part[p][0][c], out1[c] = sum_p part[p][1][c], p in order.
__global__ void __launch_bounds__(kThreads) param_reduce_kernel(const float* __restrict__ part, int64_t nparts, int C,
                                                                float* __restrict__ out0, float* __restrict__ out1) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float a = 0.f, b = 0.f;
    for (int64_t p = 0; p < nparts; ++p) {
        a += part[(p * 2) * C + c];
        b += part[(p * 2 + 1) * C + c];
    }
    out0[c] = a;
    out1[c] = b;
}

// ---- GRN (grn_cuda.cu:126-265) ------------------------------------------------------------
// y = x (1 + gamma Nx) + beta, Nx = Gx inv, Gx[b, c] = ||x[b, :, c]||, inv = 1 / (mean_c Gx + eps).
// With t[b, c] = sum_s dy x and s = gamma t:
//   dgamma = sum_b Nx t,  dbeta = sum_b sum_s dy,
//   dGx = s inv - (sum_c s Gx) inv^2 / C,
//   dx = dy (1 + gamma Nx) + dGx x / Gx   (0 where Gx = 0).
// grn_stats_bwd_kernel: CTA = (b, block of 32 channels), pixel lanes reduced in lane order.
template <typename T>
__global__ void __launch_bounds__(kThreads) grn_stats_bwd_kernel(const float* __restrict__ dy,
                                                                 const T* __restrict__ x, int S, int C,
                                                                 float* __restrict__ t_out,
                                                                 float* __restrict__ dbeta_bc) {
    const int b = blockIdx.x;
    const int c = blockIdx.y * 32 + (threadIdx.x & 31);
    const int pl = threadIdx.x >> 5;
    float t = 0.f, sb = 0.f;
    if (c < C) {
        const int64_t base = (int64_t)b * S * C + c;
        for (int s = pl; s < S; s += kThreads / 32) {
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
        t_out[(int64_t)b * C + c] = a;
        dbeta_bc[(int64_t)b * C + c] = bsum;
    }
}

// One CTA per image: dGx[b, :] from t, gamma, Gx and inv (the sum over channels in a fixed
// tree order).
__global__ void __launch_bounds__(kThreads) grn_dgx_kernel(const float* __restrict__ t, const float* __restrict__ gamma,
                                                           const float* __restrict__ gx,
                                                           const float* __restrict__ inv_den, int C,
                                                           float* __restrict__ dgx) {
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
    for (int c = threadIdx.x; c < C; c += kThreads)
        dgx[(int64_t)b * C + c] = gamma[c] * t[(int64_t)b * C + c] * inv - tot * inv * inv / (float)C;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) grn_dx_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                          const float* __restrict__ gamma, const float* __restrict__ gx,
                                                          const float* __restrict__ inv_den,
                                                          const float* __restrict__ dgx, T* __restrict__ dx, int S,
                                                          int C, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const int64_t b = i / ((int64_t)S * C);
        const float g = gx[b * C + c];
        const float nx = g * inv_den[b];
        const float xv = to_f(x[i]);
        const float igx = g > 0.f ? 1.f / g : 0.f;
        dx[i] = from_f<T>(fmaf(dy[i], fmaf(gamma[c], nx, 1.f), dgx[b * C + c] * xv * igx));
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
    for (int b = 0; b < B; ++b) {
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

int64_t dirfuse_parts(int batch, int height, int width) {
    return (int64_t)batch * (((int64_t)height * width + kPix - 1) / kPix);
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
    return dirfuse_parts(batch, height, width) * 8 * (int64_t)heads * head_dim * (int64_t)sizeof(float);
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
    const int tiles = (int)((L + kPix - 1) / kPix);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    int rc = by_dtype(io_dtype, [&](auto t) {
        using T = decltype(t);
        const dim3 grid(tiles, (C + 31) / 32, batch);
        dirfuse_bwd_kernel<T><<<grid, kThreads, 0, st>>>(grad_out, gs_b, gs_c, gs_h, gs_w, static_cast<const T*>(y),
                                                         static_cast<const T*>(x), skip, skip_per_dir ? 1 : 0, scale,
                                                         static_cast<T*>(grad_y), static_cast<T*>(grad_x), part,
                                                         heads, height, width, head_dim);
        return launch_status("vh_dirfuse_bwd");
    });
    if (rc) return rc;
    dirfuse_reduce_kernel<<<(C + kThreads - 1) / kThreads, kThreads, 0, st>>>(
        part, dirfuse_parts(batch, height, width), C, skip_per_dir ? 1 : 0, grad_scale, grad_skip);
    return launch_status("vh_dirfuse_bwd (reduce)");
}

extern "C" int64_t vh_layernorm_bwd_workspace_bytes(int64_t rows, int32_t channels) {
    if (rows <= 0 || channels <= 0) return 0;
    return ((rows + kLnRows - 1) / kLnRows) * 2 * (int64_t)channels * (int64_t)sizeof(float);
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
        const int64_t grid = (rows + kThreads / 32 - 1) / (kThreads / 32);
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
    param_reduce_kernel<<<(channels + kThreads - 1) / kThreads, kThreads, 0, st>>>(part, rblocks, channels,
                                                                                     grad_weight, grad_bias);
    return launch_status("vh_layernorm_bwd (reduce)");
}

extern "C" int64_t vh_grn_bwd_workspace_bytes(int32_t batch, int32_t channels) {
    if (batch <= 0 || channels <= 0) return 0;
    return 3 * (int64_t)batch * channels * (int64_t)sizeof(float);
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
    float* dgx = dbeta_bc + (int64_t)batch * channels;
    return by_dtype(x_dtype, [&](auto tag) {
        using T = decltype(tag);
        const T* xp = static_cast<const T*>(x);
        grn_stats_bwd_kernel<T><<<dim3(batch, (channels + 31) / 32), kThreads, 0, st>>>(grad_y, xp, (int)S, channels,
                                                                                      t, dbeta_bc);
        int r = launch_status("vh_grn_bwd (stats)");
        if (r) return r;
        grn_dgx_kernel<<<batch, kThreads, 0, st>>>(t, gamma, gx, inv_den, channels, dgx);
        if ((r = launch_status("vh_grn_bwd (dGx)"))) return r;
        const int grid = (int)std::min<int64_t>((n + kThreads - 1) / kThreads, (int64_t)sm_count() * 8);
        grn_dx_kernel<T><<<grid, kThreads, 0, st>>>(grad_y, xp, gamma, gx, inv_den, dgx, static_cast<T*>(grad_x),
                                                    (int)S, channels, n);
        if ((r = launch_status("vh_grn_bwd (dx)"))) return r;
        grn_param_kernel<<<(channels + kThreads - 1) / kThreads, kThreads, 0, st>>>(t, gx, inv_den, dbeta_bc, batch,
                                                                                   channels, grad_gamma, grad_beta);
        return launch_status("vh_grn_bwd (params)");
    });
}
