// SRNL recurrence backward, head_dim 16: one warp per chain, any chunk length.
// Included by srnl_bwd.cu (namespace vh::sbwd); same two sweeps and the same arithmetic as
// srnl_bwd_kernel, scheduled for a warp:
//   - token-parallel work (loads, projections, gates, the gate adjoint, dx, dq) runs with one
//     lane per token over tiles of 32 tokens, the records of a tile held in shared memory;
//   - the serial work is the gain recurrence G_t = alpha G_{t-1} - eff r k^T (forward) and its
//     adjoint dG_{t-1} = alpha dG_t + dr k^T (reverse), 16 x 16 matrices held 8 entries per
//     lane (lane = 2 i + h: row i, columns 8h..8h+7).  The reverse step also forms the
//     quantities that need dG_t itself (dG k, <dG, G_{t-1}>, -eff dG^T r + G_{t-1}^T dr and
//     d eff) with warp shuffles, and leaves the rest of the gate adjoint to the token-parallel
//     phase.  G_{t-1} of every token is written to the workspace by the gain recurrence and read
//     back, one token ahead, by the reverse pass.  When the whole history fits the workspace
//     budget (`full_history`), sweep A writes it for every chunk, with each chunk's final gain,
//     and sweep B does not run the gain recurrence again; otherwise sweep B recomputes each
//     chunk's history just before reversing it.
// The token-parallel phases that run once per tile (dx, the parameter adjoint) are kept as
// loops rather than unrolled: with eleven warps per SM in different phases, instruction fetch
// had been the largest stall, and the smaller code measured faster (as did a prefetch distance
// of one token over two to eight).
// Tokens past the sequence end in the last chunk are skipped: the last chunk's gain is never
// applied, so its dG is zero throughout and those tokens contribute nothing.
#pragma once

namespace wb {

constexpr int D = 16;
constexpr int SR = 3 * D + 2;  // rows of the state [M_m; M_v; M_k; e; a]
constexpr int kTile = 32;      // tokens per record tile (one per lane)
constexpr int kRS = kTile + 1; // record row stride: lane t and row i at i * kRS + t
constexpr unsigned kFull = 0xffffffffu;

// Record rows (one column per token of the tile).  In the reverse pass R_K is overwritten
// with dk~ and R_D with dv once the token's adjoint is complete.
enum : int {
    R_X = 0,
    R_QH = 16,
    R_K = 32,
    R_D = 48,
    R_DY = 64,
    R_DGK = 80,  // dG k
    R_WG = 96,   // -eff dG^T r + G_{t-1}^T dr
    R_KINV = 112,
    R_QINV,
    R_EP,
    R_AP,
    R_ETA,
    R_ALPHA,
    R_SIG,
    R_DN,
    R_CAP,
    R_TAKE0,  // 1 where eff = cap (1 - exp(-eta / cap)), 0 where the clamp limit binds
    R_EFF,
    R_KE,
    R_DAL,   // <dG, G_{t-1}>, then d(x.e)
    R_DEFF,  // d eff, then d(x.a)
    R_ROWS
};
constexpr int R_DEP = R_DAL;
constexpr int R_DAP = R_DEFF;

struct WSmem {
    float S[SR][D];  // chunk-start state
    union {
        float rec[R_ROWS][kRS];
        struct {
            float dS[SR][D + 1];
            float GT[D][D + 1];
        } m;  // between the forward and the reverse pass of a chunk
    };
};

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void stcg4(float* p, float4 v) { __stcg(reinterpret_cast<float4*>(p), v); }

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[D]) {
    float a[8], c[8];
    load8(p, a);
    load8(p + 8, c);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = a[i];
        v[8 + i] = c[i];
    }
}

// Token-parallel part of a tile: token tok0 + lane for lane < n.  FULL: every record the
// reverse pass needs; otherwise only those of the gain recurrence (k, d, alpha, eff).
template <typename XT, typename QT, bool FULL>
__device__ __forceinline__ void tile_tokens(const Params& p, WSmem& s, int64_t chain, int b, int r, int head,
                                            int64_t tok0, int n, int lane) {
    if (lane >= n) return;
    const int64_t tok = tok0 + lane;
    float (*rec)[kRS] = s.rec;
    float xv[D];
    load16(static_cast<const XT*>(p.x) + (chain * p.L + tok) * D, xv);
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
        rec[R_K + i][lane] = kk;
        rec[R_D + i][lane] = dd;
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
    rec[R_ALPHA][lane] = alpha;
    rec[R_EFF][lane] = eff;
    if constexpr (FULL) {
        float qv[D];
        float qinv = 1.f;
        if (p.q_mode == 0) {
            const int C = p.heads * D;
            load16(static_cast<const QT*>(p.q) + (((int64_t)b * p.R + r) * p.L + tok) * C + head * D, qv);
            float qs = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) qs = fmaf(qv[i], qv[i], qs);
            qinv = 1.f / fmaxf(sqrtf(qs), 1e-12f);
        } else {
            load16(static_cast<const float*>(p.q) + (chain * p.L + tok) * D, qv);
        }
        const float* dyp = p.dy + (chain * p.L + tok) * D;
#pragma unroll
        for (int i4 = 0; i4 < D / 4; ++i4) {
            const float4 g = *reinterpret_cast<const float4*>(dyp + 4 * i4);
            rec[R_DY + 4 * i4][lane] = g.x;
            rec[R_DY + 4 * i4 + 1][lane] = g.y;
            rec[R_DY + 4 * i4 + 2][lane] = g.z;
            rec[R_DY + 4 * i4 + 3][lane] = g.w;
        }
#pragma unroll
        for (int i = 0; i < D; ++i) {
            rec[R_X + i][lane] = xv[i];
            rec[R_QH + i][lane] = qv[i] * qinv;
        }
        rec[R_KINV][lane] = kinv;
        rec[R_QINV][lane] = qinv;
        rec[R_EP][lane] = ep;
        rec[R_AP][lane] = apr;
        rec[R_ETA][lane] = eta;
        rec[R_SIG][lane] = sig;
        rec[R_DN][lane] = dn;
        rec[R_CAP][lane] = cap;
        rec[R_TAKE0][lane] = (!K.spectral_clamp || eff0 <= lim) ? 1.f : 0.f;
        rec[R_KE][lane] = ke;
    }
}

// Forward gain recurrence of one chunk of n tokens from G = I (records recomputed tile by
// tile); when gseq is given, G_{t-1} of token t goes to gseq + t * 256.  G ends as G_n.
template <typename XT, typename QT>
__device__ __forceinline__ void chunk_gain_warp(const Params& p, WSmem& s, int64_t chain, int b, int r, int head,
                                                int64_t tok0, int n, float* gseq, float (&G)[8], int lane) {
    const int i = lane >> 1, h = lane & 1;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) G[jj] = (i == 8 * h + jj) ? 1.f : 0.f;
    for (int t0 = 0; t0 < n; t0 += kTile) {
        const int nt = min(kTile, n - t0);
        __syncwarp();
        tile_tokens<XT, QT, false>(p, s, chain, b, r, head, tok0 + t0, nt, lane);
        __syncwarp();
        for (int tt = 0; tt < nt; ++tt) {
            if (gseq) {
                float* gp = gseq + (int64_t)(t0 + tt) * (D * D) + lane * 8;
                stcg4(gp, make_float4(G[0], G[1], G[2], G[3]));
                stcg4(gp + 4, make_float4(G[4], G[5], G[6], G[7]));
            }
            float kk[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) kk[jj] = s.rec[R_K + 8 * h + jj][tt];
            const float di = s.rec[R_D + i][tt];
            const float al = s.rec[R_ALPHA][tt], ef = s.rec[R_EFF][tt];
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int jj = 0; jj < 8; jj += 2) {
                a0 = fmaf(G[jj], kk[jj], a0);
                a1 = fmaf(G[jj + 1], kk[jj + 1], a1);
            }
            float pr = a0 + a1;
            pr += __shfl_xor_sync(kFull, pr, 1);
            const float ri = di + pr;
            const float er = ef * ri;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) G[jj] = al * G[jj] - er * kk[jj];
        }
    }
    __syncwarp();
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// One reverse step of token tt (records of the current tile); g = G_{t-1} (this lane's 8).
// Updates dG to dG_{t-1} and writes R_DGK, R_WG, R_DAL, R_DEFF of the token.
__device__ __forceinline__ void reverse_step(WSmem& s, int tt, const float (&g)[8], float (&dG)[8], int lane) {
    const int i = lane >> 1, h = lane & 1;
    float kk[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) kk[jj] = s.rec[R_K + 8 * h + jj][tt];
    const float di = s.rec[R_D + i][tt];
    const float al = s.rec[R_ALPHA][tt], eff = s.rec[R_EFF][tt];
    // r_i = d_i + (G_{t-1} k)_i, (dG k)_i, and the lane's part of <dG, G_{t-1}>
    float p0 = 0.f, p1 = 0.f, q0 = 0.f, q1 = 0.f, dal = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; jj += 2) {
        p0 = fmaf(g[jj], kk[jj], p0);
        p1 = fmaf(g[jj + 1], kk[jj + 1], p1);
        q0 = fmaf(dG[jj], kk[jj], q0);
        q1 = fmaf(dG[jj + 1], kk[jj + 1], q1);
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) dal = fmaf(dG[jj], g[jj], dal);
    float pr = p0 + p1, dgk = q0 + q1;
    pr += __shfl_xor_sync(kFull, pr, 1);
    dgk += __shfl_xor_sync(kFull, dgk, 1);
    const float ri = di + pr;
    const float dri = -eff * dgk;
    // -eff dG[i][j] r_i + G_{t-1}[i][j] dr_i, summed over i below
    const float er = -eff * ri;
    float pv[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) pv[jj] = fmaf(g[jj], dri, er * dG[jj]);
    // dG_{t-1} = alpha dG_t + dr k^T: the only value the next step waits for
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) dG[jj] = fmaf(al, dG[jj], dri * kk[jj]);
    // d eff = -sum_i r_i (dG k)_i (one lane per row)
    const float de = warp_allsum(h == 0 ? -ri * dgk : 0.f);
    dal = warp_allsum(dal);
    // Column sums of pv over the 16 rows (lanes of equal h): halve the values held per lane at
    // each exchange; the lane ends with column 8h + 4 b4 + 2 b3 + b2.
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float u[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float send = b4 ? pv[m] : pv[m + 4];
        const float keep = b4 ? pv[m + 4] : pv[m];
        u[m] = keep + __shfl_xor_sync(kFull, send, 16);
    }
    float w2[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const float send = b3 ? u[m] : u[m + 2];
        const float keep = b3 ? u[m + 2] : u[m];
        w2[m] = keep + __shfl_xor_sync(kFull, send, 8);
    }
    float z;
    {
        const float send = b2 ? w2[0] : w2[1];
        const float keep = b2 ? w2[1] : w2[0];
        z = keep + __shfl_xor_sync(kFull, send, 4);
    }
    z += __shfl_xor_sync(kFull, z, 2);
    const int jcol = 8 * h + (b4 ? 4 : 0) + (b3 ? 2 : 0) + (b2 ? 1 : 0);
    if (h == 0) s.rec[R_DGK + i][tt] = dgk;
    if ((lane & 2) == 0) s.rec[R_WG + jcol][tt] = z;
    if (lane == 0) {
        s.rec[R_DAL][tt] = dal;
        s.rec[R_DEFF][tt] = de;
    }
}

// Token-parallel rest of the adjoint (lane = token): the gates, the key normalization and
// k = v + d into dk~ (R_K), dv (R_D), d(x.e), d(x.a) (R_DEP, R_DAP).
__device__ __forceinline__ void gate_adjoint(WSmem& s, const SrnlConsts& K, int tt, bool zero) {
    float (*rec)[kRS] = s.rec;
    if (zero) {
#pragma unroll
        for (int j = 0; j < D; ++j) {
            rec[R_K + j][tt] = 0.f;
            rec[R_D + j][tt] = 0.f;
        }
        rec[R_DEP][tt] = 0.f;
        rec[R_DAP][tt] = 0.f;
        return;
    }
    const float eff = rec[R_EFF][tt], al = rec[R_ALPHA][tt];
    const float d_eff = rec[R_DEFF][tt], dal_direct = rec[R_DAL][tt];
    const bool take0 = rec[R_TAKE0][tt] != 0.f;
    const float d_eff0 = take0 ? d_eff : 0.f, d_lim = take0 ? 0.f : d_eff;
    const float ke = rec[R_KE][tt];
    const float kem = fmaxf(ke, 1e-20f);
    float d_alpha = dal_direct + d_lim * K.spectral_factor / kem;
    const float d_ke = (!take0 && ke > 1e-20f) ? -d_lim * K.spectral_factor * al / (kem * kem) : 0.f;
    const float cap = rec[R_CAP][tt], u = rec[R_ETA][tt] / cap;
    const float em = expf(-u);
    const float d_eta = d_eff0 * em;
    const float d_cap = d_eff0 * ((1.f - em) - u * em);
    const float dn = rec[R_DN][tt];
    const float den = dn + 1e-6f;
    d_alpha += d_cap * (-K.injection_margin / den);
    const float d_dn = d_cap * (-cap / den);
    const float ep_raw = rec[R_EP][tt], ap_raw = rec[R_AP][tt];
    const float epc = fminf(10.f, fmaxf(-10.f, ep_raw));
    const float sp = 1.f / (1.f + expf(-epc));  // softplus'
    const float ep_in = (ep_raw >= -10.f && ep_raw <= 10.f) ? 1.f : 0.f;
    const float ap_in = (ap_raw >= -10.f && ap_raw <= 10.f) ? 1.f : 0.f;
    const float sg = rec[R_SIG][tt];
    const float d_ap = ap_in * d_alpha * (1.f - K.min_retention) * sg * (1.f - sg);
    const float d_ep = ep_in * d_eta * K.step_scale * sp;
    const float ddn = d_dn / dn;  // d(dn) / dn, applied to each d_j
    float dk[D], kv[D], kdk = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) {
        const float dr = -eff * rec[R_DGK + j][tt];
        const float dd = fmaf(ddn, rec[R_D + j][tt], dr);
        kv[j] = rec[R_K + j][tt];
        dk[j] = rec[R_WG + j][tt] + dd + 2.f * d_ke * kv[j];
        rec[R_D + j][tt] = -dd;
        kdk = fmaf(kv[j], dk[j], kdk);
    }
    const float kinv = rec[R_KINV][tt];
#pragma unroll
    for (int j = 0; j < D; ++j) rec[R_K + j][tt] = kinv * (dk[j] - kv[j] * kdk);
    rec[R_DEP][tt] = d_ep;
    rec[R_DAP][tt] = d_ap;
}

__device__ __forceinline__ void load_ring(const float* gseq, int64_t t, int lane, float (&g)[8]) {
    const float* gp = gseq + (int64_t)t * (D * D) + lane * 8;
    const float4 a = ldcg4(gp), c = ldcg4(gp + 4);
    g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
    g[4] = c.x; g[5] = c.y; g[6] = c.z; g[7] = c.w;
}

template <typename XT, typename QT>
__global__ void __launch_bounds__(32, 11) srnl_bwd_warp_kernel(const Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WSmem& s = *reinterpret_cast<WSmem*>(smem_raw);
    const int lane = threadIdx.x;
    const int64_t chain = blockIdx.x;  // ((b * R + r) * heads + head)
    const int head = (int)(chain % p.heads);
    const int r = (int)((chain / p.heads) % p.R);
    const int b = (int)(chain / ((int64_t)p.heads * p.R));
    const int Lc = p.chunk[r];
    const int nch = (p.L + Lc - 1) / Lc;
    float* states = p.states + chain * (int64_t)p.nchunks_max * SR * D;
    float* gseq = p.gseq + chain * p.gseq_stride;
    // full: sweep A keeps G_{t-1} of every token of the sequence and each chunk's final gain,
    // and sweep B reads them instead of running the gain recurrence a second time.
    const bool full = p.full_history != 0;
    float* gend = p.gend + chain * (int64_t)p.nchunks_max * (D * D);
    const int i = lane >> 1, h = lane & 1;
    const int rb = lane >> 4, col = lane & 15;  // element layout of dS: rows rb + 2k, column col

    // ---- A: forward sweep, chunk-start states --------------------------------------------
    {
        const int64_t sidx = p.mem_per_chain ? chain : (int64_t)r * p.heads + head;
        for (int e = lane; e < SR * D; e += 32) {
            const int row = e / D, c = e % D;
            float v;
            if (row < D) v = p.Mm[(sidx * D + row) * D + c];
            else if (row < 2 * D) v = p.Mv[(sidx * D + row - D) * D + c];
            else if (row < 3 * D) v = p.Mk[(sidx * D + row - 2 * D) * D + c];
            else if (row == 3 * D) v = p.Me[sidx * D + c];
            else v = p.Ma[sidx * D + c];
            s.S[row][c] = v;
        }
        __syncwarp();
    }
    for (int c = 0; c < nch; ++c) {
        for (int e = lane; e < SR * D; e += 32) states[(int64_t)c * SR * D + e] = s.S[e / D][e % D];
        if (c + 1 == nch) break;
        float G[8];
        chunk_gain_warp<XT, QT>(p, s, chain, b, r, head, (int64_t)c * Lc, Lc,
                                full ? gseq + (int64_t)c * Lc * (D * D) : nullptr, G, lane);
        if (full) {
            float* ge = gend + (int64_t)c * (D * D) + lane * 8;
            stcg4(ge, make_float4(G[0], G[1], G[2], G[3]));
            stcg4(ge + 4, make_float4(G[4], G[5], G[6], G[7]));
        }
        // S <- S G
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) s.m.GT[i][8 * h + jj] = G[jj];
        __syncwarp();
        float nv[SR * D / 32];
#pragma unroll
        for (int k = 0; k < SR * D / 32; ++k) {
            const int e = lane + 32 * k, row = e / D, cc = e % D;
            float a = 0.f;
#pragma unroll
            for (int l = 0; l < D; ++l) a = fmaf(s.S[row][l], s.m.GT[l][cc], a);
            nv[k] = a;
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < SR * D / 32; ++k) {
            const int e = lane + 32 * k;
            s.S[e / D][e % D] = nv[k];
        }
        __syncwarp();
    }

    // ---- B: backward sweep ---------------------------------------------------------------
    float dS[SR * D / 32];  // element (rb + 2k, col)
#pragma unroll
    for (int k = 0; k < SR * D / 32; ++k) dS[k] = 0.f;
    const SrnlConsts& K = p.k;
    for (int c = nch - 1; c >= 0; --c) {
        const int64_t tok0 = (int64_t)c * Lc;
        const int n = (int)(p.L - tok0 < Lc ? p.L - tok0 : Lc);
        const bool last = c + 1 == nch;  // its gain is never applied: dG = 0 throughout
        __syncwarp();
        for (int e = lane; e < SR * D; e += 32) s.S[e / D][e % D] = states[(int64_t)c * SR * D + e];
        __syncwarp();
        float dG[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) dG[jj] = 0.f;
        const float* gseq_c = full ? gseq + (int64_t)c * Lc * (D * D) : gseq;
        if (!last) {
            float G[8];
            if (full) {
                load_ring(gend + (int64_t)c * (D * D), 0, lane, G);  // G_T kept by sweep A
            } else {
                chunk_gain_warp<XT, QT>(p, s, chain, b, r, head, tok0, n, gseq, G, lane);
            }
            // dG_T = S_c^T dS_{c+1};  dS_c starts as dS_{c+1} G_T^T
#pragma unroll
            for (int k = 0; k < SR * D / 32; ++k) s.m.dS[rb + 2 * k][col] = dS[k];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) s.m.GT[i][8 * h + jj] = G[jj];
            __syncwarp();
            for (int row = 0; row < SR; ++row) {
                const float sv = s.S[row][i];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) dG[jj] = fmaf(sv, s.m.dS[row][8 * h + jj], dG[jj]);
            }
#pragma unroll
            for (int k = 0; k < SR * D / 32; ++k) {
                const int row = rb + 2 * k;
                float a = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) a = fmaf(s.m.dS[row][j], s.m.GT[col][j], a);
                dS[k] = a;
            }
            __syncwarp();
        }
        // Reverse pass, last tile first.
        const int ntiles = (n + kTile - 1) / kTile;
        for (int tile = ntiles - 1; tile >= 0; --tile) {
            const int t0 = tile * kTile;
            const int nt = min(kTile, n - t0);
            tile_tokens<XT, QT, true>(p, s, chain, b, r, head, tok0 + t0, nt, lane);
            __syncwarp();
            if (!last) {
                float gc[8], gn[8];
                load_ring(gseq_c, t0 + nt - 1, lane, gc);
#pragma unroll 1
                for (int tt = nt - 1; tt >= 0; --tt) {
                    if (tt > 0) load_ring(gseq_c, t0 + tt - 1, lane, gn);
                    reverse_step(s, tt, gc, dG, lane);
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) gc[jj] = gn[jj];
                }
            }
            __syncwarp();
            if (lane < nt) gate_adjoint(s, K, lane, last);
            __syncwarp();
            // Parameter adjoint: dS += sum_t [dy q^T; dv x^T; dk~ x^T; d(x.e) x; d(x.a) x]
#pragma unroll 1
            for (int tt = 0; tt < nt; ++tt) {
                const float xj = s.rec[R_X + col][tt], qj = s.rec[R_QH + col][tt];
#pragma unroll
                for (int k = 0; k < 8; ++k) dS[k] = fmaf(s.rec[R_DY + rb + 2 * k][tt], qj, dS[k]);
#pragma unroll
                for (int k = 0; k < 8; ++k) dS[8 + k] = fmaf(s.rec[R_D + rb + 2 * k][tt], xj, dS[8 + k]);
#pragma unroll
                for (int k = 0; k < 8; ++k) dS[16 + k] = fmaf(s.rec[R_K + rb + 2 * k][tt], xj, dS[16 + k]);
                dS[24] = fmaf(s.rec[rb ? R_DAP : R_DEP][tt], xj, dS[24]);
            }
            // dx_t = M_v^T dv + M_k^T dk~ + d(x.e) e + d(x.a) a;  dq from dq^ = M_m^T dy
            if (lane < nt) {
                const int64_t tok = tok0 + t0 + lane;
                const float dep = s.rec[R_DEP][lane], dap = s.rec[R_DAP][lane];
                float dv[D], dkt[D], dy[D];
#pragma unroll
                for (int q = 0; q < D; ++q) {
                    dv[q] = s.rec[R_D + q][lane];
                    dkt[q] = s.rec[R_K + q][lane];
                    dy[q] = s.rec[R_DY + q][lane];
                }
                float* dxp = p.dx + (chain * p.L + tok) * D;
#pragma unroll 1
                for (int j4 = 0; j4 < D / 4; ++j4) {
                    float o[4];
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int j = 4 * j4 + m;
                        float a = dep * s.S[3 * D][j];
                        a = fmaf(dap, s.S[3 * D + 1][j], a);
#pragma unroll
                        for (int q = 0; q < D; ++q) {
                            a = fmaf(s.S[D + q][j], dv[q], a);
                            a = fmaf(s.S[2 * D + q][j], dkt[q], a);
                        }
                        o[m] = a;
                    }
                    *reinterpret_cast<float4*>(dxp + 4 * j4) = make_float4(o[0], o[1], o[2], o[3]);
                }
                float dqh[D], dot = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) {
                    float a = 0.f;
#pragma unroll
                    for (int q = 0; q < D; ++q) a = fmaf(s.S[q][j], dy[q], a);
                    dqh[j] = a;
                    dot = fmaf(a, s.rec[R_QH + j][lane], dot);
                }
                float* dst;
                if (p.q_mode == 0) {
                    const float qi = s.rec[R_QINV][lane];
                    const bool clamped = qi > 9.999e11f;
                    dst = p.dq + (((int64_t)b * p.R + r) * p.L + tok) * (p.heads * D) + head * D;
#pragma unroll
                    for (int j = 0; j < D; ++j)
                        dqh[j] = clamped ? dqh[j] * qi : (dqh[j] - s.rec[R_QH + j][lane] * dot) * qi;
                } else {
                    dst = p.dq + (chain * p.L + tok) * D;
                }
#pragma unroll
                for (int j4 = 0; j4 < D / 4; ++j4)
                    *reinterpret_cast<float4*>(dst + 4 * j4) =
                        make_float4(dqh[4 * j4], dqh[4 * j4 + 1], dqh[4 * j4 + 2], dqh[4 * j4 + 3]);
            }
            __syncwarp();
        }
    }
#pragma unroll
    for (int k = 0; k < SR * D / 32; ++k) p.dS[chain * SR * D + (rb + 2 * k) * D + col] = dS[k];
}

}  // namespace wb
