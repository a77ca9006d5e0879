// Query normalization (+ relayout) and direction restoration/fusion kernels, with their
// C entry points.  Both are HBM-bound; every thread moves whole 4-channel vectors.
#include "abi_util.h"
#include "common.cuh"

namespace vh {

// ---- query normalization: [B,R,L,C] -> fp32 [B,R,heads,L,D] (query_normalization.cu:136-178)
// One thread per (b, r, head, l) vector, l fastest so the fp32 output rows are written
// contiguously; the input rows are whole D-element (>= 8-byte) segments.
template <int D, typename T>
__global__ void __launch_bounds__(256) qnorm_kernel(const T* __restrict__ q, float* __restrict__ out,
                                                    float* __restrict__ inv_norm, int B, int R, int L,
                                                    int heads) {
    const int64_t n = (int64_t)B * R * heads * L;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    const int l = (int)(idx % L);
    const int64_t rest = idx / L;
    const int head = (int)(rest % heads);
    const int64_t br = rest / heads;  // b * R + r
    const int C = heads * D;
    const T* src = q + (br * L + l) * C + (int64_t)head * D;
    float v[D];
#pragma unroll
    for (int i = 0; i < D; i += 4) {
        const float4 f = load4(src + i);
        v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) ss = fmaf(v[i], v[i], ss);
    const float inv = 1.f / fmaxf(sqrtf(ss), 1e-12f);
    float* dst = out + idx * D;
#pragma unroll
    for (int i = 0; i < D; i += 4)
        store4(dst + i, make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv));
    if (inv_norm) inv_norm[(br * L + l) * heads + head] = inv;
}

// ---- direction fusion (direction_fusion.cu:11-65) ------------------------------------------
// CTA = (b, head, tile of TP consecutive row-major pixels).  Each thread builds the fused
// 4-channel vector of one pixel from the four scans; channels-last output is written
// directly, NCHW output is transposed through shared memory so every channel row of TP
// pixels is one contiguous store.
constexpr int kFuseTP = 64;

template <int D, typename T, bool CL>
__global__ void __launch_bounds__(256) dirfuse_kernel(const T* __restrict__ y, const T* __restrict__ x,
                                                      const float* __restrict__ skip, int skip_per_dir,
                                                      const float* __restrict__ scale,
                                                      float* __restrict__ out, int heads, int H, int W) {
    constexpr int G4 = D / 4;
    __shared__ float tileT[D][kFuseTP + 1];
    const int64_t L = (int64_t)H * W;
    const int C = heads * D;
    const int tiles = (int)((L + kFuseTP - 1) / kFuseTP);
    const int tile = blockIdx.x % tiles;
    const int head = (blockIdx.x / tiles) % heads;
    const int b = blockIdx.x / (tiles * heads);
    const int64_t pix0 = (int64_t)tile * kFuseTP;
    for (int it = threadIdx.x; it < kFuseTP * G4; it += blockDim.x) {
        const int g = it % G4, k = it / G4;
        const int64_t pix = pix0 + k;
        if (pix >= L) continue;
        const int h = (int)(pix / W), w = (int)(pix % W);
        const int64_t lhw = pix, lwh = (int64_t)w * H + h;
        const int64_t ls[4] = {lhw, L - 1 - lhw, lwh, L - 1 - lwh};
        const int c0 = head * D + g * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int64_t off = ((((int64_t)b * 4 + d) * heads + head) * L + ls[d]) * D + g * 4;
            const float4 yv = load4(y + off), xv = load4(x + off);
            const float* sk = skip + (skip_per_dir ? d * C : 0) + c0;
            const float* sc = scale + d * C + c0;
            acc.x += sc[0] * (yv.x + sk[0] * xv.x);
            acc.y += sc[1] * (yv.y + sk[1] * xv.y);
            acc.z += sc[2] * (yv.z + sk[2] * xv.z);
            acc.w += sc[3] * (yv.w + sk[3] * xv.w);
        }
        if constexpr (CL) {
            store4(out + ((int64_t)b * L + pix) * C + c0, acc);
        } else {
            tileT[g * 4 + 0][k] = acc.x;
            tileT[g * 4 + 1][k] = acc.y;
            tileT[g * 4 + 2][k] = acc.z;
            tileT[g * 4 + 3][k] = acc.w;
        }
    }
    if constexpr (!CL) {
        __syncthreads();
        for (int it = threadIdx.x; it < D * kFuseTP; it += blockDim.x) {
            const int k = it % kFuseTP, ch = it / kFuseTP;
            const int64_t pix = pix0 + k;
            if (pix < L) out[((int64_t)b * C + head * D + ch) * L + pix] = tileT[ch][k];
        }
    }
}

template <typename T>
int qnorm_dispatch(int D, const void* q, float* out, float* inv, int B, int R, int L, int heads,
                   cudaStream_t st) {
    const int64_t n = (int64_t)B * R * heads * L;
    const dim3 grid((unsigned)((n + 255) / 256));
    const T* qp = static_cast<const T*>(q);
    switch (D) {
        case 4: qnorm_kernel<4, T><<<grid, 256, 0, st>>>(qp, out, inv, B, R, L, heads); break;
        case 8: qnorm_kernel<8, T><<<grid, 256, 0, st>>>(qp, out, inv, B, R, L, heads); break;
        case 16: qnorm_kernel<16, T><<<grid, 256, 0, st>>>(qp, out, inv, B, R, L, heads); break;
        case 32: qnorm_kernel<32, T><<<grid, 256, 0, st>>>(qp, out, inv, B, R, L, heads); break;
        case 64: qnorm_kernel<64, T><<<grid, 256, 0, st>>>(qp, out, inv, B, R, L, heads); break;
        default: return fail(VH_E_HEADDIM, "unsupported head_dim %d", D);
    }
    return launch_status("qnorm");
}

template <typename T, bool CL>
int dirfuse_dispatch_cl(int D, const void* y, const void* x, const float* skip, int spd,
                        const float* scale, float* out, int B, int heads, int H, int W, cudaStream_t st) {
    const int64_t L = (int64_t)H * W;
    const int64_t tiles = (L + kFuseTP - 1) / kFuseTP;
    const dim3 grid((unsigned)(tiles * heads * B));
    const T* yp = static_cast<const T*>(y);
    const T* xp = static_cast<const T*>(x);
    switch (D) {
        case 4: dirfuse_kernel<4, T, CL><<<grid, 256, 0, st>>>(yp, xp, skip, spd, scale, out, heads, H, W); break;
        case 8: dirfuse_kernel<8, T, CL><<<grid, 256, 0, st>>>(yp, xp, skip, spd, scale, out, heads, H, W); break;
        case 16: dirfuse_kernel<16, T, CL><<<grid, 256, 0, st>>>(yp, xp, skip, spd, scale, out, heads, H, W); break;
        case 32: dirfuse_kernel<32, T, CL><<<grid, 256, 0, st>>>(yp, xp, skip, spd, scale, out, heads, H, W); break;
        case 64: dirfuse_kernel<64, T, CL><<<grid, 256, 0, st>>>(yp, xp, skip, spd, scale, out, heads, H, W); break;
        default: return fail(VH_E_HEADDIM, "unsupported head_dim %d", D);
    }
    return launch_status("dirfuse");
}

template <typename T>
int dirfuse_dispatch(int cl, int D, const void* y, const void* x, const float* skip, int spd,
                     const float* scale, float* out, int B, int heads, int H, int W, cudaStream_t st) {
    return cl ? dirfuse_dispatch_cl<T, true>(D, y, x, skip, spd, scale, out, B, heads, H, W, st)
              : dirfuse_dispatch_cl<T, false>(D, y, x, skip, spd, scale, out, B, heads, H, W, st);
}

}  // namespace vh

using namespace vh;

extern "C" int vh_qnorm_fwd(const void* q_raw, int32_t q_dtype, float* out, float* inv_norm,
                            int32_t batch, int32_t dirs, int32_t length, int32_t heads,
                            int32_t head_dim, vh_stream_t stream) {
    clear_error();
    if (!q_raw || !out) return fail(VH_E_ARG, "vh_qnorm_fwd: null pointer argument");
    if (!dtype_ok(q_dtype)) return fail(VH_E_DTYPE, "vh_qnorm_fwd: bad dtype");
    if (!head_dim_ok(head_dim)) return fail(VH_E_HEADDIM, "Unsupported qnorm head dimension %d", head_dim);
    if (batch <= 0 || dirs <= 0 || length <= 0 || heads <= 0)
        return fail(VH_E_SHAPE, "vh_qnorm_fwd: sizes must be positive");
    if (!aligned(q_raw, q_dtype == VH_F32 ? 16 : 8) || !aligned(out, 16))
        return fail(VH_E_ALIGN, "vh_qnorm_fwd: misaligned pointers");
    if ((int64_t)batch * dirs * heads * length > ((int64_t)1 << 40))
        return fail(VH_E_RANGE, "vh_qnorm_fwd: too many vectors");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (q_dtype) {
        case VH_F32: return qnorm_dispatch<float>(head_dim, q_raw, out, inv_norm, batch, dirs, length, heads, st);
        case VH_BF16: return qnorm_dispatch<__nv_bfloat16>(head_dim, q_raw, out, inv_norm, batch, dirs, length, heads, st);
        default: return qnorm_dispatch<__half>(head_dim, q_raw, out, inv_norm, batch, dirs, length, heads, st);
    }
}

extern "C" int vh_dirfuse_fwd(const void* y, const void* x, int32_t io_dtype, const float* skip,
                              int32_t skip_per_dir, const float* scale, float* out,
                              int32_t channels_last, int32_t batch, int32_t heads, int32_t height,
                              int32_t width, int32_t head_dim, vh_stream_t stream) {
    clear_error();
    if (!y || !x || !skip || !scale || !out) return fail(VH_E_ARG, "vh_dirfuse_fwd: null pointer argument");
    if (!dtype_ok(io_dtype)) return fail(VH_E_DTYPE, "vh_dirfuse_fwd: bad dtype");
    if (!head_dim_ok(head_dim)) return fail(VH_E_HEADDIM, "unsupported head_dim %d", head_dim);
    if (batch <= 0 || heads <= 0 || height <= 0 || width <= 0)
        return fail(VH_E_SHAPE, "Invalid shape for vh_dirfuse_fwd");
    const size_t va = io_dtype == VH_F32 ? 16 : 8;
    if (!aligned(y, va) || !aligned(x, va) || !aligned(out, 16))
        return fail(VH_E_ALIGN, "vh_dirfuse_fwd: misaligned pointers");
    const int64_t tiles = ((int64_t)height * width + kFuseTP - 1) / kFuseTP;
    if (tiles * heads * batch >= ((int64_t)1 << 31)) return fail(VH_E_RANGE, "vh_dirfuse_fwd: grid too large");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int cl = channels_last != 0, spd = skip_per_dir != 0;
    switch (io_dtype) {
        case VH_F32: return dirfuse_dispatch<float>(cl, head_dim, y, x, skip, spd, scale, out, batch, heads, height, width, st);
        case VH_BF16: return dirfuse_dispatch<__nv_bfloat16>(cl, head_dim, y, x, skip, spd, scale, out, batch, heads, height, width, st);
        default: return dirfuse_dispatch<__half>(cl, head_dim, y, x, skip, spd, scale, out, batch, heads, height, width, st);
    }
}
