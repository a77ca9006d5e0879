// LayerScale residual add of the block (residual.py:30-204):
//   out[b, s, c] = residual + branch * gamma[c] * drop[b]        (fp32, channels-last)
// and its backward,
//   d residual = d out,  d branch = d out * gamma[c] * drop[b],
//   d gamma[c] = sum over (b, s) of d out * branch * drop[b].
// Both passes are HBM-bound streams over [rows = B * S, C].  d gamma is summed per CTA over a
// fixed block of rows (row lanes added in lane order), then over the row blocks in order
// (reduce_parts_kernel in backward.cu), so it is bit-reproducible.
#include <algorithm>
#include <climits>

#include "abi_util.h"
#include "common.cuh"

namespace vh {
namespace bwd {
// out[q][c] = sum over p in order of part[p][q][c] (backward.cu).
int reduce_parts(const float* part, int64_t nparts, int nq, int C, float* out, cudaStream_t st);
}  // namespace bwd

namespace res {

constexpr int kThreads = 256;
constexpr int kMinRowsPerPart = 128;
constexpr int64_t kMaxParts = 1024;

// Rows summed by one CTA of the backward: at least 128, and at most 1024 partial rows.
inline int64_t rows_per_part(int64_t rows) {
    return std::max<int64_t>(kMinRowsPerPart, (rows + kMaxParts - 1) / kMaxParts);
}

// V channels per thread (4 where C % 4 == 0).  The forward CTA covers `rows_per_cta` whole
// rows; thread i of the tile handles channel group i % (C / V) of row i / (C / V), so the
// division is 32-bit and the row's drop scale is one load per group.
template <typename RT, typename BT, int V>
__global__ void __launch_bounds__(kThreads) residual_fwd_kernel(const RT* __restrict__ residual,
                                                                const BT* __restrict__ branch,
                                                                const float* __restrict__ gamma,
                                                                const float* __restrict__ drop,
                                                                float* __restrict__ out, int64_t rows, int C,
                                                                int64_t spatial, int rows_per_cta) {
    const int groups = C / V;
    const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
    const int nrows = (int)std::min<int64_t>(rows_per_cta, rows - row0);
    const int tile = nrows * groups;
    for (int i = threadIdx.x; i < tile; i += kThreads) {
        const int rl = i / groups;
        const int c = (i - rl * groups) * V;
        const int64_t r = row0 + rl;
        const float m = drop[r / spatial];
        const int64_t off = r * C + c;
        if constexpr (V == 4) {
            const float4 a = load4(residual + off), bv = load4(branch + off);
            const float4 g = *reinterpret_cast<const float4*>(gamma + c);
            float4 o;
            o.x = fmaf(bv.x * g.x, m, a.x);
            o.y = fmaf(bv.y * g.y, m, a.y);
            o.z = fmaf(bv.z * g.z, m, a.z);
            o.w = fmaf(bv.w * g.w, m, a.w);
            store4(out + off, o);
        } else {
            out[off] = fmaf(to_f(branch[off]) * gamma[c], m, to_f(residual[off]));
        }
    }
}

// CTA = (block of `rpp` rows, block of `cgroups` channel groups).  Thread t: channel
// group t % cgroups, row lane t / cgroups; the row lanes' d gamma sums are added in lane
// order and written as the block's partial row.
template <typename BT, int V>
__global__ void __launch_bounds__(kThreads) residual_bwd_kernel(const float* __restrict__ dout,
                                                                const BT* __restrict__ branch,
                                                                const float* __restrict__ gamma,
                                                                const float* __restrict__ drop,
                                                                BT* __restrict__ dbranch,
                                                                float* __restrict__ part, int64_t rows, int C,
                                                                int64_t spatial, int cgroups, int64_t rpp) {
    __shared__ float red[kThreads][V];
    const int lanes = kThreads / cgroups;
    const int q = threadIdx.x % cgroups, rl = threadIdx.x / cgroups;
    const int c = (blockIdx.y * cgroups + q) * V;
    const bool live = rl < lanes && c < C;
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.f;
    if (live) {
        float g[V];
#pragma unroll
        for (int v = 0; v < V; ++v) g[v] = gamma[c + v];
        const int64_t r1 = std::min<int64_t>(rows, (int64_t)(blockIdx.x + 1) * rpp);
        int64_t r = (int64_t)blockIdx.x * rpp + rl;
        int64_t bi = r / spatial, bend = (bi + 1) * spatial;  // image of row r, and its end
        for (; r < r1; r += lanes) {
            while (r >= bend) {
                ++bi;
                bend += spatial;
            }
            const float m = drop[bi];
            const int64_t off = r * C + c;
            if constexpr (V == 4) {
                const float4 d = *reinterpret_cast<const float4*>(dout + off);
                const float4 bv = load4(branch + off);
                acc[0] = fmaf(d.x * bv.x, m, acc[0]);
                acc[1] = fmaf(d.y * bv.y, m, acc[1]);
                acc[2] = fmaf(d.z * bv.z, m, acc[2]);
                acc[3] = fmaf(d.w * bv.w, m, acc[3]);
                store4(dbranch + off, make_float4(d.x * (g[0] * m), d.y * (g[1] * m), d.z * (g[2] * m), d.w * (g[3] * m)));
            } else {
                const float d = dout[off];
                acc[0] = fmaf(d * to_f(branch[off]), m, acc[0]);
                dbranch[off] = from_f<BT>(d * (g[0] * m));
            }
        }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) red[threadIdx.x][v] = acc[v];
    __syncthreads();
    if (rl == 0 && c < C) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float s = red[q][v];
            for (int k = 1; k < lanes; ++k) s += red[k * cgroups + q][v];
            part[(int64_t)blockIdx.x * C + c + v] = s;
        }
    }
}

template <typename F>
int by_dtype(int dt, F&& f) {
    switch (dt) {
        case VH_F32: return f(float{});
        case VH_BF16: return f(__nv_bfloat16{});
        default: return f(__half{});
    }
}

// Channel groups per backward CTA: all of them up to 64 (at least 4 row lanes).
inline int bwd_cgroups(int C, int V) { return std::min(C / V, 64); }

}  // namespace res
}  // namespace vh

using namespace vh;
using namespace vh::res;

extern "C" int vh_residual_add_fwd(const void* residual, int32_t residual_dtype, const void* branch,
                                   int32_t branch_dtype, const float* gamma, const float* drop_scale, float* out,
                                   int32_t batch, int64_t spatial, int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!residual || !branch || !gamma || !drop_scale || !out)
        return fail(VH_E_ARG, "vh_residual_add_fwd: null pointer argument");
    if (!dtype_ok(residual_dtype) || !dtype_ok(branch_dtype)) return fail(VH_E_DTYPE, "vh_residual_add_fwd: bad dtype");
    if (batch <= 0 || spatial <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_residual_add_fwd: sizes must be positive");
    const int64_t rows = (int64_t)batch * spatial;
    if (rows * channels > ((int64_t)1 << 40)) return fail(VH_E_RANGE, "vh_residual_add_fwd: too many elements");
    const bool vec = channels % 4 == 0 && aligned(residual, 4 * dtype_size(residual_dtype)) &&
                     aligned(branch, 4 * dtype_size(branch_dtype)) && aligned(gamma, 16) && aligned(out, 16);
    const int V = vec ? 4 : 1;
    const int groups = channels / V;
    // About eight groups per thread per CTA; a CTA holds at least one whole row.
    const int rows_per_cta = std::max(1, (8 * kThreads) / groups);
    if ((int64_t)rows_per_cta * groups > INT32_MAX) return fail(VH_E_RANGE, "vh_residual_add_fwd: rows too wide");
    const int64_t grid = (rows + rows_per_cta - 1) / rows_per_cta;
    if (grid > INT32_MAX) return fail(VH_E_RANGE, "vh_residual_add_fwd: too many rows");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return by_dtype(residual_dtype, [&](auto rt) {
        using RT = decltype(rt);
        return by_dtype(branch_dtype, [&](auto bt) {
            using BT = decltype(bt);
            if (vec)
                residual_fwd_kernel<RT, BT, 4><<<(unsigned)grid, kThreads, 0, st>>>(
                    static_cast<const RT*>(residual), static_cast<const BT*>(branch), gamma, drop_scale, out, rows,
                    channels, spatial, rows_per_cta);
            else
                residual_fwd_kernel<RT, BT, 1><<<(unsigned)grid, kThreads, 0, st>>>(
                    static_cast<const RT*>(residual), static_cast<const BT*>(branch), gamma, drop_scale, out, rows,
                    channels, spatial, rows_per_cta);
            return launch_status("vh_residual_add_fwd");
        });
    });
}

extern "C" int64_t vh_residual_add_bwd_workspace_bytes(int64_t rows, int32_t channels) {
    if (rows <= 0 || channels <= 0) return 0;
    const int64_t rpp = rows_per_part(rows);
    return ((rows + rpp - 1) / rpp) * (int64_t)channels * (int64_t)sizeof(float);
}

extern "C" int vh_residual_add_bwd(const float* grad_out, const void* branch, int32_t branch_dtype,
                                   const float* gamma, const float* drop_scale, void* grad_branch,
                                   float* grad_gamma, void* workspace, int64_t workspace_bytes, int32_t batch,
                                   int64_t spatial, int32_t channels, vh_stream_t stream) {
    clear_error();
    if (!grad_out || !branch || !gamma || !drop_scale || !grad_branch || !grad_gamma || !workspace)
        return fail(VH_E_ARG, "vh_residual_add_bwd: null pointer argument");
    if (!dtype_ok(branch_dtype)) return fail(VH_E_DTYPE, "vh_residual_add_bwd: bad dtype");
    if (batch <= 0 || spatial <= 0 || channels <= 0) return fail(VH_E_SHAPE, "vh_residual_add_bwd: sizes must be positive");
    const int64_t rows = (int64_t)batch * spatial;
    if (workspace_bytes < vh_residual_add_bwd_workspace_bytes(rows, channels))
        return fail(VH_E_ARG, "vh_residual_add_bwd: workspace too small");
    const int64_t rpp = rows_per_part(rows);
    const int64_t parts = (rows + rpp - 1) / rpp;
    if (rows * channels > ((int64_t)1 << 40) || parts > INT32_MAX)
        return fail(VH_E_RANGE, "vh_residual_add_bwd: too many elements");
    const bool vec = channels % 4 == 0 && aligned(grad_out, 16) && aligned(branch, 4 * dtype_size(branch_dtype)) &&
                     aligned(grad_branch, 4 * dtype_size(branch_dtype)) && aligned(gamma, 16);
    const int V = vec ? 4 : 1;
    const int cg = bwd_cgroups(channels, V);
    const int cblocks = (channels / V + cg - 1) / cg;
    if (cblocks > 65535) return fail(VH_E_RANGE, "vh_residual_add_bwd: too many channels");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    int rc = by_dtype(branch_dtype, [&](auto bt) {
        using BT = decltype(bt);
        const dim3 grid((unsigned)parts, (unsigned)cblocks);
        if (vec)
            residual_bwd_kernel<BT, 4><<<grid, kThreads, 0, st>>>(grad_out, static_cast<const BT*>(branch), gamma,
                                                                  drop_scale, static_cast<BT*>(grad_branch), part,
                                                                  rows, channels, spatial, cg, rpp);
        else
            residual_bwd_kernel<BT, 1><<<grid, kThreads, 0, st>>>(grad_out, static_cast<const BT*>(branch), gamma,
                                                                  drop_scale, static_cast<BT*>(grad_branch), part,
                                                                  rows, channels, spatial, cg, rpp);
        return launch_status("vh_residual_add_bwd");
    });
    if (rc) return rc;
    return vh::bwd::reduce_parts(part, parts, 1, channels, grad_gamma, st);
}
