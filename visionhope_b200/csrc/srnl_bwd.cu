// SRNL recurrence backward (training) for packed sequences, replacing the reference's
// srnl_backward (models/srnl_core/csrc/chunk.cu:511-1057, chunk.py:286-359, 507-588).
//
// One CTA per chain (b, r, head), two sweeps:
//   A  forward over the chunks from the initial memories, storing every chunk-start state
//      S_c = [M_m; M_v; M_k; e; a] ((3D+2) x D, fp32) in the workspace;
//   B  backward over the chunks, last first.  For chunk c it recomputes the token quantities
//      from S_c (projections, gates) and the gain recurrence, keeping G_{t-1} of every token in
//      the workspace, then runs the adjoint of
//        r_t = d_t + G_{t-1} k_t,   G_t = alpha_t G_{t-1} - eff_t r_t k_t^T
//      from dG_T = S_c^T dS_{c+1} (S_{c+1} = S_c G_T) back to the first token, through the
//      gates (eff = min(cap (1 - exp(-eta/cap)), clamp limit), cap, eta = step softplus(x.e),
//      alpha = min_ret + (1 - min_ret) sigmoid(x.a + bias), the key normalization) into
//      d k~, d v, d(x.e), d(x.a) per token; then, once per chunk, the parameter adjoint
//      dS_c = dS_{c+1} G_T^T + sum_t [dy_t q_t^T; dv_t x_t^T; dk~_t x_t^T; d(x.e)_t x_t; d(x.a)_t x_t]
//      and the input gradients dx_t, dq_t.
// The forward arithmetic is the forward kernels' (the same gate function), so the recomputed
// states are the ones the forward used.  Every sum runs in a fixed order: gradients are
// bit-reproducible.  Shared (per direction and head) memories get their gradient as the sum
// over the batch of the per-chain ones, added in batch order by a second kernel.
#include <algorithm>
#include <cstdlib>
#include <climits>

#include "abi_util.h"
#include "common.cuh"
#include "srnl_scan.cuh"

namespace vh {
namespace sbwd {

constexpr int kT = 128;     // threads per CTA
constexpr int kMaxT = 64;   // tokens per chunk (the reference's MAX_CHUNK, chunk.py:18)

struct Params {
    const float* Mm;
    const float* Mv;
    const float* Mk;
    const float* Me;
    const float* Ma;
    int mem_per_chain;
    const void* x;   // [B, R, heads, L, D]
    const void* q;   // raw [B, R, L, C] (q_mode 0) or unit-norm fp32 [B, R, heads, L, D] (1)
    int q_mode;
    const float* dy;  // [B, R, heads, L, D]
    float* dx;        // [B, R, heads, L, D]
    float* dq;        // q's layout
    float* dS;        // [chains][(3D+2) D]: gradient of the chain's initial state
    float* states;    // [chains][nchunks_max][(3D+2) D]
    float* gseq;      // [chains][gseq_stride]: G_{t-1} of each token (one chunk, or all: full_history)
    int64_t gseq_stride;
    int full_history;  // head_dim 16: sweep A keeps every token's G_{t-1} and each chunk's G_T
    float* gend;       // [chains][nchunks_max][D D]: G_T of each chunk (full_history)
    int B, R, heads, L, nchunks_max;
    int chunk[4];
    SrnlConsts k;
};

// Per-token quantities of one chunk, recomputed from S_c (shared memory).
template <int D>
struct Tok {
    float x[kMaxT][D];
    float qh[kMaxT][D];   // normalized query
    float k[kMaxT][D];    // normalized key
    float d[kMaxT][D];    // k - v
    float r[kMaxT][D];    // d + G_{t-1} k
    float kinv[kMaxT], qinv[kMaxT], ep_raw[kMaxT], ap_raw[kMaxT], eta[kMaxT], alpha[kMaxT], sig[kMaxT];
    float dn[kMaxT], cap[kMaxT], eff0[kMaxT], lim[kMaxT], eff[kMaxT], ke[kMaxT];
    // adjoints produced by the reverse token loop
    float dkt[kMaxT][D];  // d k~
    float dv[kMaxT][D];
    float dep[kMaxT], dap[kMaxT];
};

template <int D>
struct Smem {
    static constexpr int SR = 3 * D + 2;
    float S[SR][D];     // chunk-start state
    float G[D][D];      // gain (forward) / its adjoint dG (backward)
    float Gp[D][D];     // G_{t-1} of the token being reversed
    float dSn[SR][D];   // adjoint of the next chunk's state
    float vec[4][D];    // per-token vectors: dGk, dG^T r, dr, dk
    float red[kT / 32];
    Tok<D> tok;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kT / 32; ++w) s += red[w];
    return s;
}

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i) { return to_f(p[i]); }

// Token-parallel part of a chunk from S (one thread per token): inputs, projections and gates.
template <int D, typename XT, typename QT>
__device__ void chunk_tokens(const Params& p, Smem<D>& s, int64_t chain, int b, int r, int head, int c,
                             int Lc) {
    Tok<D>& tk = s.tok;
    const int C = p.heads * D;
    for (int t = threadIdx.x; t < Lc; t += kT) {
        const int64_t tok = (int64_t)c * Lc + t;
        const bool live = tok < p.L;
        float xv[D], qv[D];
#pragma unroll
        for (int i = 0; i < D; ++i) {
            xv[i] = live ? ld(static_cast<const XT*>(p.x), (chain * p.L + tok) * D + i) : 0.f;
            if (p.q_mode == 0)
                qv[i] = live ? ld(static_cast<const QT*>(p.q), (((int64_t)b * p.R + r) * p.L + tok) * C + head * D + i) : 0.f;
            else
                qv[i] = live ? ld(static_cast<const QT*>(p.q), (chain * p.L + tok) * D + i) : 0.f;
        }
        float qinv = 1.f;
        if (p.q_mode == 0) {
            float qs = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) qs = fmaf(qv[i], qv[i], qs);
            qinv = 1.f / fmaxf(sqrtf(qs), 1e-12f);
        }
        float kt[D], vv[D], kn = 0.f, ep = 0.f, ap = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) {
            float a = 0.f, bq = 0.f;
#pragma unroll
            for (int j = 0; j < D; ++j) {
                a = fmaf(s.S[2 * D + i][j], xv[j], a);
                bq = fmaf(s.S[D + i][j], xv[j], bq);
            }
            kt[i] = a;
            vv[i] = bq;
            kn = fmaf(a, a, kn);
            ep = fmaf(xv[i], s.S[3 * D][i], ep);
            ap = fmaf(xv[i], s.S[3 * D + 1][i], ap);
        }
        const float kinv = key_inv_norm(kn);
        float ke = 0.f, dn2 = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) {
            const float kk = kt[i] * kinv;
            const float dd = kk - vv[i];
            tk.x[t][i] = xv[i];
            tk.qh[t][i] = qv[i] * qinv;
            tk.k[t][i] = kk;
            tk.d[t][i] = dd;
            ke = fmaf(kk, kk, ke);
            dn2 = fmaf(dd, dd, dn2);
        }
        // The gate arithmetic of token_gate_scalars, with the intermediates the adjoint needs.
        const SrnlConsts& K = p.k;
        const float epc = fminf(10.f, fmaxf(-10.f, ep));
        const float apr = ap + K.retention_bias;
        const float apc = fminf(10.f, fmaxf(-10.f, apr));
        const float eta = K.step_scale * (epc > 20.f ? epc : __logf(1.f + __expf(epc)));
        const float sig = __fdividef(1.f, 1.f + __expf(-apc));
        const float alpha = K.min_retention + (1.f - K.min_retention) * sig;
        const float dsq = dn2 + 1e-12f;
        const float dn = dsq * rsqrtf(dsq);
        const float cap = __fdividef(K.injection_margin * (1.f - alpha), dn + 1e-6f);
        const float eff0 = cap * (-expm1f(-__fdividef(eta, cap)));
        float lim = INFINITY, eff = eff0;
        if (K.spectral_clamp) {
            lim = nextafterf(__fdividef(K.spectral_factor * alpha, fmaxf(ke, 1e-20f)), 0.f);
            eff = fminf(eff0, lim);
        }
        tk.kinv[t] = kinv;
        tk.qinv[t] = qinv;
        tk.ep_raw[t] = ep;
        tk.ap_raw[t] = apr;
        tk.eta[t] = eta;
        tk.alpha[t] = alpha;
        tk.sig[t] = sig;
        tk.dn[t] = dn;
        tk.cap[t] = cap;
        tk.eff0[t] = eff0;
        tk.lim[t] = lim;
        tk.eff[t] = eff;
        tk.ke[t] = ke;
    }
    __syncthreads();
}

// The chunk's gain recurrence from G = I; when `keep`, G_{t-1} of every token goes to gseq
// and r_t to the token record.
template <int D>
__device__ void chunk_gain(Smem<D>& s, int Lc, float* gseq, bool keep) {
    Tok<D>& tk = s.tok;
    for (int e = threadIdx.x; e < D * D; e += kT) s.G[e / D][e % D] = (e / D == e % D) ? 1.f : 0.f;
    __syncthreads();
    for (int t = 0; t < Lc; ++t) {
        if (threadIdx.x < D) {
            const int i = threadIdx.x;
            float a = tk.d[t][i];
#pragma unroll
            for (int j = 0; j < D; ++j) a = fmaf(s.G[i][j], tk.k[t][j], a);
            tk.r[t][i] = a;
        }
        if (keep)
            for (int e = threadIdx.x; e < D * D; e += kT) gseq[(int64_t)t * D * D + e] = s.G[e / D][e % D];
        __syncthreads();
        const float al = tk.alpha[t], ef = tk.eff[t];
        for (int e = threadIdx.x; e < D * D; e += kT) {
            const int i = e / D, j = e % D;
            s.G[i][j] = al * s.G[i][j] - ef * tk.r[t][i] * tk.k[t][j];
        }
        __syncthreads();
    }
}

template <int D, typename XT, typename QT>
__global__ void __launch_bounds__(kT) srnl_bwd_kernel(const Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem<D>& s = *reinterpret_cast<Smem<D>*>(smem_raw);
    constexpr int SR = Smem<D>::SR;
    const int64_t chain = blockIdx.x;  // ((b * R + r) * heads + head)
    const int head = (int)(chain % p.heads);
    const int r = (int)((chain / p.heads) % p.R);
    const int b = (int)(chain / ((int64_t)p.heads * p.R));
    const int Lc = p.chunk[r];
    const int nch = (p.L + Lc - 1) / Lc;
    float* states = p.states + chain * (int64_t)p.nchunks_max * SR * D;
    float* gseq = p.gseq + chain * p.gseq_stride;
    Tok<D>& tk = s.tok;

    // ---- A: forward sweep, chunk-start states --------------------------------------------
    {
        const int64_t sidx = p.mem_per_chain ? chain : (int64_t)r * p.heads + head;
        for (int e = threadIdx.x; e < SR * D; e += kT) {
            const int row = e / D, col = e % D;
            float v;
            if (row < D) v = p.Mm[(sidx * D + row) * D + col];
            else if (row < 2 * D) v = p.Mv[(sidx * D + row - D) * D + col];
            else if (row < 3 * D) v = p.Mk[(sidx * D + row - 2 * D) * D + col];
            else if (row == 3 * D) v = p.Me[sidx * D + col];
            else v = p.Ma[sidx * D + col];
            s.S[row][col] = v;
        }
        __syncthreads();
    }
    for (int c = 0; c < nch; ++c) {
        for (int e = threadIdx.x; e < SR * D; e += kT) states[(int64_t)c * SR * D + e] = s.S[e / D][e % D];
        if (c + 1 == nch) break;
        chunk_tokens<D, XT, QT>(p, s, chain, b, r, head, c, Lc);
        chunk_gain<D>(s, Lc, gseq, false);
        // S <- S G (fp32)
        float nv[(SR * D + kT - 1) / kT];
#pragma unroll
        for (int k = 0; k < (SR * D + kT - 1) / kT; ++k) {
            const int e = threadIdx.x + k * kT;
            float a = 0.f;
            if (e < SR * D) {
                const int row = e / D, col = e % D;
#pragma unroll
                for (int l = 0; l < D; ++l) a = fmaf(s.S[row][l], s.G[l][col], a);
            }
            nv[k] = a;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < (SR * D + kT - 1) / kT; ++k) {
            const int e = threadIdx.x + k * kT;
            if (e < SR * D) s.S[e / D][e % D] = nv[k];
        }
        __syncthreads();
    }

    // ---- B: backward sweep -----------------------------------------------------------------
    for (int e = threadIdx.x; e < SR * D; e += kT) s.dSn[e / D][e % D] = 0.f;
    __syncthreads();
    const SrnlConsts& K = p.k;
    for (int c = nch - 1; c >= 0; --c) {
        for (int e = threadIdx.x; e < SR * D; e += kT) s.S[e / D][e % D] = states[(int64_t)c * SR * D + e];
        __syncthreads();
        chunk_tokens<D, XT, QT>(p, s, chain, b, r, head, c, Lc);
        chunk_gain<D>(s, Lc, gseq, true);  // s.G = G_T
        // dG_T = S_c^T dS_{c+1} into Gp (scratch), then dS_c starts as dS_{c+1} G_T^T.
        for (int e = threadIdx.x; e < D * D; e += kT) {
            const int l = e / D, j = e % D;
            float a = 0.f;
            for (int row = 0; row < SR; ++row) a = fmaf(s.S[row][l], s.dSn[row][j], a);
            s.Gp[l][j] = a;
        }
        float nd[(SR * D + kT - 1) / kT];
#pragma unroll
        for (int k = 0; k < (SR * D + kT - 1) / kT; ++k) {
            const int e = threadIdx.x + k * kT;
            float a = 0.f;
            if (e < SR * D) {
                const int row = e / D, l = e % D;
#pragma unroll
                for (int j = 0; j < D; ++j) a = fmaf(s.dSn[row][j], s.G[l][j], a);
            }
            nd[k] = a;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < (SR * D + kT - 1) / kT; ++k) {
            const int e = threadIdx.x + k * kT;
            if (e < SR * D) s.dSn[e / D][e % D] = nd[k];
        }
        for (int e = threadIdx.x; e < D * D; e += kT) s.G[e / D][e % D] = s.Gp[e / D][e % D];  // G := dG
        __syncthreads();

        // Reverse token loop: s.G holds dG_t.
        for (int t = Lc - 1; t >= 0; --t) {
            for (int e = threadIdx.x; e < D * D; e += kT) s.Gp[e / D][e % D] = gseq[(int64_t)t * D * D + e];
            __syncthreads();
            // dGk = dG k, dG^T r, <dG, G_{t-1}>
            float part = 0.f;
            for (int e = threadIdx.x; e < D * D; e += kT) part = fmaf(s.G[e / D][e % D], s.Gp[e / D][e % D], part);
            if (threadIdx.x < D) {
                const int i = threadIdx.x;
                float a = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) a = fmaf(s.G[i][j], tk.k[t][j], a);
                s.vec[0][i] = a;
            } else if (threadIdx.x >= 64 && threadIdx.x < 64 + D) {
                const int j = threadIdx.x - 64;
                float a = 0.f;
#pragma unroll
                for (int i = 0; i < D; ++i) a = fmaf(s.G[i][j], tk.r[t][i], a);
                s.vec[1][j] = a;
            }
            const float dal_direct = block_sum(part, s.red);  // includes a barrier
            const float eff = tk.eff[t], al = tk.alpha[t];
            // dr = -eff dGk;  dk = -eff dG^T r + G_{t-1}^T dr
            if (threadIdx.x < D) s.vec[2][threadIdx.x] = -eff * s.vec[0][threadIdx.x];
            __syncthreads();
            float d_eff = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) d_eff = fmaf(-tk.r[t][i], s.vec[0][i], d_eff);
            if (threadIdx.x < D) {
                const int j = threadIdx.x;
                float a = -eff * s.vec[1][j];
#pragma unroll
                for (int i = 0; i < D; ++i) a = fmaf(s.Gp[i][j], s.vec[2][i], a);
                s.vec[3][j] = a;
            }
            // dG_{t-1} = alpha dG + dr k^T
            __syncthreads();
            for (int e = threadIdx.x; e < D * D; e += kT) {
                const int i = e / D, j = e % D;
                s.G[i][j] = al * s.G[i][j] + s.vec[2][i] * tk.k[t][j];
            }
            // Gate adjoint (warp 0; the vectors by lane, the scalars redundantly per lane).
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                const bool take0 = !K.spectral_clamp || tk.eff0[t] <= tk.lim[t];
                const float d_eff0 = take0 ? d_eff : 0.f, d_lim = take0 ? 0.f : d_eff;
                const float kem = fmaxf(tk.ke[t], 1e-20f);
                float d_alpha = dal_direct + d_lim * K.spectral_factor / kem;
                const float d_ke = (!take0 && tk.ke[t] > 1e-20f) ? -d_lim * K.spectral_factor * al / (kem * kem) : 0.f;
                const float cap = tk.cap[t], u = tk.eta[t] / cap;
                const float em = expf(-u);
                const float d_eta = d_eff0 * em;
                const float d_cap = d_eff0 * ((1.f - em) - u * em);
                const float den = tk.dn[t] + 1e-6f;
                d_alpha += d_cap * (-K.injection_margin / den);
                const float d_dn = d_cap * (-cap / den);
                const float epc = fminf(10.f, fmaxf(-10.f, tk.ep_raw[t]));
                const float sp = 1.f / (1.f + expf(-epc));  // softplus'
                const float ep_in = (tk.ep_raw[t] >= -10.f && tk.ep_raw[t] <= 10.f) ? 1.f : 0.f;
                const float ap_in = (tk.ap_raw[t] >= -10.f && tk.ap_raw[t] <= 10.f) ? 1.f : 0.f;
                const float sg = tk.sig[t];
                const float d_ap = ap_in * d_alpha * (1.f - K.min_retention) * sg * (1.f - sg);
                const float d_ep = ep_in * d_eta * K.step_scale * sp;
                // dd = dr + d_dn d / dn;  dk += dd + 2 d_ke k;  dv = -dd;  dk~ = kinv (dk - k (k.dk))
                float dkv[(D + 31) / 32], kv[(D + 31) / 32], kdk = 0.f;
#pragma unroll
                for (int m = 0; m < (D + 31) / 32; ++m) {
                    const int i = lane + 32 * m;
                    dkv[m] = 0.f;
                    kv[m] = 0.f;
                    if (i < D) {
                        const float dd = s.vec[2][i] + d_dn * tk.d[t][i] / tk.dn[t];
                        kv[m] = tk.k[t][i];
                        dkv[m] = s.vec[3][i] + dd + 2.f * d_ke * kv[m];
                        tk.dv[t][i] = -dd;
                        kdk = fmaf(kv[m], dkv[m], kdk);
                    }
                }
                kdk = warp_sum(kdk);
                const float kinv = tk.kinv[t];
#pragma unroll
                for (int m = 0; m < (D + 31) / 32; ++m) {
                    const int i = lane + 32 * m;
                    if (i < D) tk.dkt[t][i] = kinv * (dkv[m] - kv[m] * kdk);
                }
                if (lane == 0) {
                    tk.dep[t] = d_ep;
                    tk.dap[t] = d_ap;
                }
            }
            __syncthreads();
        }
        // dG_{-1} (adjoint of G = I) does not propagate.  Parameter adjoint of this chunk and
        // the input gradients.
        for (int e = threadIdx.x; e < SR * D; e += kT) {
            const int row = e / D, j = e % D;
            float a = s.dSn[row][j];
            if (row < D) {  // dM_m += sum_t dy_t q_t^T
                for (int t = 0; t < Lc; ++t) {
                    const int64_t tok = (int64_t)c * Lc + t;
                    if (tok < p.L) a = fmaf(p.dy[(chain * p.L + tok) * D + row], tk.qh[t][j], a);
                }
            } else if (row < 2 * D) {
                for (int t = 0; t < Lc; ++t) a = fmaf(tk.dv[t][row - D], tk.x[t][j], a);
            } else if (row < 3 * D) {
                for (int t = 0; t < Lc; ++t) a = fmaf(tk.dkt[t][row - 2 * D], tk.x[t][j], a);
            } else if (row == 3 * D) {
                for (int t = 0; t < Lc; ++t) a = fmaf(tk.dep[t], tk.x[t][j], a);
            } else {
                for (int t = 0; t < Lc; ++t) a = fmaf(tk.dap[t], tk.x[t][j], a);
            }
            s.dSn[row][j] = a;  // each element is read and written by this thread only
        }
        // dx_t = M_v^T dv + M_k^T dk~ + d(x.e) e + d(x.a) a;  dq from dq^ = M_m^T dy.
        const int C = p.heads * D;
        for (int e = threadIdx.x; e < Lc * D; e += kT) {
            const int t = e / D, j = e % D;
            const int64_t tok = (int64_t)c * Lc + t;
            if (tok >= p.L) continue;
            float a = tk.dep[t] * s.S[3 * D][j];
            a = fmaf(tk.dap[t], s.S[3 * D + 1][j], a);
#pragma unroll
            for (int i = 0; i < D; ++i) {
                a = fmaf(s.S[D + i][j], tk.dv[t][i], a);
                a = fmaf(s.S[2 * D + i][j], tk.dkt[t][i], a);
            }
            p.dx[(chain * p.L + tok) * D + j] = a;
        }
        for (int t = threadIdx.x; t < Lc; t += kT) {
            const int64_t tok = (int64_t)c * Lc + t;
            if (tok >= p.L) continue;
            float dqh[D], dot = 0.f;
#pragma unroll
            for (int j = 0; j < D; ++j) {
                float a = 0.f;
#pragma unroll
                for (int i = 0; i < D; ++i) a = fmaf(s.S[i][j], p.dy[(chain * p.L + tok) * D + i], a);
                dqh[j] = a;
                dot = fmaf(a, tk.qh[t][j], dot);
            }
            if (p.q_mode == 0) {
                const float qi = tk.qinv[t];
                const bool clamped = qi > 9.999e11f;
                float* dst = p.dq + (((int64_t)b * p.R + r) * p.L + tok) * C + head * D;
#pragma unroll
                for (int j = 0; j < D; ++j) dst[j] = clamped ? dqh[j] * qi : (dqh[j] - tk.qh[t][j] * dot) * qi;
            } else {
                float* dst = p.dq + (chain * p.L + tok) * D;
#pragma unroll
                for (int j = 0; j < D; ++j) dst[j] = dqh[j];
            }
        }
        __syncthreads();
    }
    for (int e = threadIdx.x; e < SR * D; e += kT) p.dS[chain * SR * D + e] = s.dSn[e / D][e % D];
}

// Gradients of shared memories: the per-chain ones summed over the batch, in batch order, and
// split into the five parameter tensors ([R, heads, D, D] x 3, [R, heads, D] x 2).
// Grid (slot, block of 64 state entries); each thread sums one entry over the batch with
// eight loads in flight.
constexpr int kMemThreads = 64;

template <int D>
__global__ void __launch_bounds__(kMemThreads) srnl_bwd_mem_kernel(const float* __restrict__ dS, int B, int R,
                                                                   int heads, int per_chain, float* __restrict__ dMm,
                                                                   float* __restrict__ dMv, float* __restrict__ dMk,
                                                                   float* __restrict__ dMe, float* __restrict__ dMa) {
    constexpr int SR = 3 * D + 2;
    const int64_t slot = blockIdx.x;  // per_chain: chain; else r * heads + head
    const int e = blockIdx.y * kMemThreads + threadIdx.x;
    if (e >= SR * D) return;
    const int nb = per_chain ? 1 : B;
    const int64_t stride = (int64_t)R * heads * SR * D;  // from one image's chain to the next
    const float* src = dS + slot * SR * D + e;
    float a = 0.f;
    int bb = 0;
    for (; bb + 8 <= nb; bb += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = src[(int64_t)(bb + u) * stride];
#pragma unroll
        for (int u = 0; u < 8; ++u) a += v[u];
    }
    for (; bb < nb; ++bb) a += src[(int64_t)bb * stride];
    const int row = e / D, col = e % D;
    if (row < D) dMm[(slot * D + row) * D + col] = a;
    else if (row < 2 * D) dMv[(slot * D + row - D) * D + col] = a;
    else if (row < 3 * D) dMk[(slot * D + row - 2 * D) * D + col] = a;
    else if (row == 3 * D) dMe[slot * D + col] = a;
    else dMa[slot * D + col] = a;
}

#include "srnl_bwd_warp.cuh"

}  // namespace sbwd
}  // namespace vh

using namespace vh;
using namespace vh::sbwd;

namespace {

// The whole G_{t-1} history is kept (head_dim 16) while it stays within this many bytes: 6 GiB,
// or VHOPE_SRNL_BWD_HISTORY_BYTES (0: always recompute each chunk's history, the smaller
// workspace).  Read at each call, so the workspace query and the call agree while it is unchanged.
int64_t history_cap() {
    const char* e = std::getenv("VHOPE_SRNL_BWD_HISTORY_BYTES");
    return e && *e ? std::atoll(e) : ((int64_t)6 << 30);
}

int max_chunks(const vh_srnl_sequence_bwd_args* a) {
    int n = 1;
    for (int r = 0; r < a->dirs; ++r) n = std::max(n, (a->length + a->chunk[r] - 1) / a->chunk[r]);
    return n;
}

int64_t max_chunk_len(const vh_srnl_sequence_bwd_args* a) {
    int64_t t = 1;
    for (int r = 0; r < a->dirs; ++r) t = std::max<int64_t>(t, std::min(a->chunk[r], a->length));
    return t;
}

template <int D>
bool full_history(const vh_srnl_sequence_bwd_args* a) {
    if (D != 16) return false;
    const int64_t chains = (int64_t)a->batch * a->dirs * a->heads;
    const int64_t per_chain = (int64_t)max_chunks(a) * max_chunk_len(a) * D * D * (int64_t)sizeof(float);
    const int64_t cap = history_cap();
    return cap > 0 && chains <= cap / per_chain;  // no overflow of chains x per_chain
}

// Floats of G_{t-1} history per chain: every token (full history), the longest chunk (head_dim
// 16, the warp kernel, takes any chunk length) or kMaxT tokens.
template <int D>
int64_t gseq_floats(const vh_srnl_sequence_bwd_args* a) {
    if (D != 16) return (int64_t)kMaxT * D * D;
    const int64_t t = max_chunk_len(a);
    return (full_history<D>(a) ? max_chunks(a) * t : t) * D * D;
}

template <int D>
int64_t bwd_workspace(const vh_srnl_sequence_bwd_args* a, int* nmax) {
    const int n = max_chunks(a);
    if (nmax) *nmax = n;
    const int64_t chains = (int64_t)a->batch * a->dirs * a->heads;
    const int64_t SR = 3 * D + 2;
    const int64_t gend = full_history<D>(a) ? (int64_t)n * D * D : 0;
    return chains * ((int64_t)n * SR * D + gseq_floats<D>(a) + SR * D + gend) * (int64_t)sizeof(float);
}

int64_t gseq_floats_d(const vh_srnl_sequence_bwd_args* a) {
    switch (a->head_dim) {
        case 4: return gseq_floats<4>(a);
        case 8: return gseq_floats<8>(a);
        case 16: return gseq_floats<16>(a);
        default: return gseq_floats<32>(a);
    }
}

int64_t bwd_workspace_d(const vh_srnl_sequence_bwd_args* a, int* nmax) {
    switch (a->head_dim) {
        case 4: return bwd_workspace<4>(a, nmax);
        case 8: return bwd_workspace<8>(a, nmax);
        case 16: return bwd_workspace<16>(a, nmax);
        default: return bwd_workspace<32>(a, nmax);
    }
}

template <int D, typename XT, typename QT>
int launch_bwd(const vh_srnl_sequence_bwd_args* a, Params p, cudaStream_t st) {
    const int64_t chains = (int64_t)a->batch * a->dirs * a->heads;
    if constexpr (D == 16) {
        const size_t smem = sizeof(wb::WSmem);
        const void* fn = reinterpret_cast<const void*>(&wb::srnl_bwd_warp_kernel<XT, QT>);
        if (!ensure_smem_attr(fn, smem))
            return fail(VH_E_DEVICE, "vh_srnl_sequence_bwd: cannot reserve %zu bytes of shared memory", smem);
        wb::srnl_bwd_warp_kernel<XT, QT><<<(unsigned)chains, 32, smem, st>>>(p);
    } else {
        const size_t smem = sizeof(Smem<D>);
        const void* fn = reinterpret_cast<const void*>(&srnl_bwd_kernel<D, XT, QT>);
        if (!ensure_smem_attr(fn, smem))
            return fail(VH_E_DEVICE, "vh_srnl_sequence_bwd: cannot reserve %zu bytes of shared memory", smem);
        srnl_bwd_kernel<D, XT, QT><<<(unsigned)chains, kT, smem, st>>>(p);
    }
    int rc = launch_status("vh_srnl_sequence_bwd");
    if (rc) return rc;
    const int64_t slots = a->mem.per_chain ? chains : (int64_t)a->dirs * a->heads;
    constexpr int SRD = (3 * D + 2) * D;
    srnl_bwd_mem_kernel<D><<<dim3((unsigned)slots, (SRD + kMemThreads - 1) / kMemThreads), kMemThreads, 0, st>>>(
        p.dS, a->batch, a->dirs, a->heads, a->mem.per_chain ? 1 : 0, a->grad_m, a->grad_v, a->grad_k, a->grad_eta,
        a->grad_alpha);
    return launch_status("vh_srnl_sequence_bwd (memories)");
}

template <typename XT, typename QT>
int dispatch_bwd(const vh_srnl_sequence_bwd_args* a, Params p, cudaStream_t st) {
    switch (a->head_dim) {
        case 4: return launch_bwd<4, XT, QT>(a, p, st);
        case 8: return launch_bwd<8, XT, QT>(a, p, st);
        case 16: return launch_bwd<16, XT, QT>(a, p, st);
        default: return launch_bwd<32, XT, QT>(a, p, st);
    }
}

const char* check_bwd(const vh_srnl_sequence_bwd_args* a) {
    if (!a || !a->mem.m || !a->mem.v || !a->mem.k || !a->mem.eta || !a->mem.alpha || !a->x || !a->q ||
        !a->grad_y || !a->grad_x || !a->grad_q || !a->grad_m || !a->grad_v || !a->grad_k || !a->grad_eta ||
        !a->grad_alpha)
        return "null pointer argument";
    return nullptr;
}

}  // namespace

extern "C" int64_t vh_srnl_sequence_bwd_workspace_bytes(const vh_srnl_sequence_bwd_args* a) {
    if (!a || a->batch <= 0 || a->dirs <= 0 || a->dirs > 4 || a->heads <= 0 || a->length <= 0) return 0;
    if (a->length > (1 << 30)) return 0;  // beyond the supported range (the call refuses it too)
    if (a->head_dim != 4 && a->head_dim != 8 && a->head_dim != 16 && a->head_dim != 32) return 0;
    for (int r = 0; r < a->dirs; ++r)
        if (a->chunk[r] <= 0) return 0;
    return bwd_workspace_d(a, nullptr);
}

extern "C" int vh_srnl_sequence_bwd(const vh_srnl_sequence_bwd_args* a, void* workspace, int64_t workspace_bytes,
                                    vh_stream_t stream) {
    clear_error();
    if (const char* why = check_bwd(a)) return fail(VH_E_ARG, "vh_srnl_sequence_bwd: %s", why);
    if (!workspace) return fail(VH_E_ARG, "vh_srnl_sequence_bwd: null workspace");
    if (!dtype_ok(a->x_dtype)) return fail(VH_E_DTYPE, "vh_srnl_sequence_bwd: bad dtype");
    if (a->q_mode == 0 && a->q_dtype != a->x_dtype)
        return fail(VH_E_DTYPE, "SRNL raw queries must match the input dtype");
    if (a->q_mode == 1 && a->q_dtype != VH_F32) return fail(VH_E_DTYPE, "SRNL normalized queries must be fp32");
    if (a->q_mode != 0 && a->q_mode != 1) return fail(VH_E_ARG, "vh_srnl_sequence_bwd: bad q_mode");
    if (a->head_dim != 4 && a->head_dim != 8 && a->head_dim != 16 && a->head_dim != 32)
        return fail(VH_E_HEADDIM, "SRNL backward supports head_dim 4, 8, 16 and 32 (got %d)", a->head_dim);
    if (a->dirs != 1 && a->dirs != 2 && a->dirs != 4)
        return fail(VH_E_SHAPE, "SRNL supports 1, 2 or 4 directions (got %d)", a->dirs);
    if (a->batch <= 0 || a->heads <= 0 || a->length <= 0)
        return fail(VH_E_SHAPE, "SRNL requires nonempty batches and sequences");
    for (int r = 0; r < a->dirs; ++r) {
        if (a->chunk[r] <= 0) return fail(VH_E_SHAPE, "SRNL chunk length must be positive");
        if (a->chunk[r] > kMaxT && a->head_dim != 16)
            return fail(VH_E_RANGE, "chunk_size=%d exceeds MAX_CHUNK=%d in the SRNL backward for head_dim %d",
                        a->chunk[r], kMaxT, a->head_dim);
    }
    const int64_t chains = (int64_t)a->batch * a->dirs * a->heads;
    if (chains > INT32_MAX || (int64_t)a->length > ((int64_t)1 << 30))
        return fail(VH_E_RANGE, "vh_srnl_sequence_bwd: sizes exceed the supported range");
    int nmax = 1;
    const int64_t need = bwd_workspace_d(a, &nmax);
    if (workspace_bytes < need) return fail(VH_E_ARG, "vh_srnl_sequence_bwd: workspace too small (%lld < %lld bytes)",
                                            (long long)workspace_bytes, (long long)need);
    const int D = a->head_dim;
    const int64_t SR = 3 * D + 2;
    Params p{};
    p.Mm = a->mem.m; p.Mv = a->mem.v; p.Mk = a->mem.k; p.Me = a->mem.eta; p.Ma = a->mem.alpha;
    p.mem_per_chain = a->mem.per_chain != 0;
    p.x = a->x; p.q = a->q; p.q_mode = a->q_mode;
    p.dy = a->grad_y; p.dx = a->grad_x; p.dq = a->grad_q;
    float* ws = static_cast<float*>(workspace);
    p.states = ws;
    p.gseq = p.states + chains * (int64_t)nmax * SR * D;
    p.gseq_stride = gseq_floats_d(a);
    p.dS = p.gseq + chains * p.gseq_stride;
    p.full_history = a->head_dim == 16 && full_history<16>(a) ? 1 : 0;
    p.gend = p.dS + chains * SR * D;  // used (and sized) only with full_history
    p.B = a->batch; p.R = a->dirs; p.heads = a->heads; p.L = a->length; p.nchunks_max = nmax;
    for (int r = 0; r < 4; ++r) p.chunk[r] = r < a->dirs ? a->chunk[r] : 1;
    const vh_srnl_consts& c = a->consts;
    p.k = {c.step_scale, c.min_retention, c.retention_bias, c.injection_margin, c.spectral_factor, c.spectral_clamp};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->q_mode == 1) {
        switch (a->x_dtype) {
            case VH_F32: return dispatch_bwd<float, float>(a, p, st);
            case VH_BF16: return dispatch_bwd<__nv_bfloat16, float>(a, p, st);
            default: return dispatch_bwd<__half, float>(a, p, st);
        }
    }
    switch (a->x_dtype) {
        case VH_F32: return dispatch_bwd<float, float>(a, p, st);
        case VH_BF16: return dispatch_bwd<__nv_bfloat16, __nv_bfloat16>(a, p, st);
        default: return dispatch_bwd<__half, __half>(a, p, st);
    }
}
