// SRNL chunked-scan kernels (sm_100a).
//
// One CTA runs `nch` independent chains (a chain = one (batch, direction, head) scan) in
// lockstep over their chunks.  Every chunk has three phases:
//   P1 token-parallel (one thread per token): q normalization, y = M_m q, k~ = M_k x,
//      v = M_v x, the key normalization, the learning-rate / retention gates, the soft
//      injection cap and the spectral clamp -- all from the chunk-start state, all
//      reductions in-thread (models/srnl_core/csrc/inference_recurrence.cuh:40-90,
//      chunk.cu:344-405, memory.cuh:219-233);
//   P2 sequential gain recurrence, one thread per row of G:
//      r = (k - v) + G k,  G <- alpha G - eta_eff r k^T   (inference_recurrence.cuh:92-106);
//   P3 boundary refresh of the stacked state S = [M_m; M_v; M_k; e^T; a^T] (3D+2 rows):
//      S <- S G   (inference_recurrence.cuh:110-135).
// Token tiles of each chunk are prefetched into shared memory with cp.async one tile ahead.
//
// Kinds:
//   kKindRows / kKindCols: the fused spatial operator (fused.cu:307-351 +
//      parallel_line.cuh:2-59).  A CTA holds (b, head) pairs of scans {0,1} (rows pass) or
//      {2,3} (columns pass) and writes weight_d * (y_d + skip_d x_d) straight into the fp32
//      output.  The rows pass runs first; every pixel is touched exactly twice per pass and
//      the order of the two touches is a fixed function of (chunk, tile), so the result is
//      deterministic: the first touch stores, the second adds, coincident touches are
//      combined by the even direction.
//   kKindSeq: packed sequences (fused.cu:93-179, chunk.cu:252-509, lines.cu:3-237), y out.
#pragma once

#include "common.cuh"

namespace vh {

constexpr int kScanThreads = 128;
enum ScanKind { kKindRows = 0, kKindCols = 1, kKindSeq = 2 };

struct ScanParams {
    const float* Mm;
    const float* Mv;
    const float* Mk;
    const float* Me;
    const float* Ma;
    int mem_per_chain;
    const void* x;
    const void* q;
    int64_t xb, xd, xt, xh;  // element strides: batch, direction slab, token, head
    int64_t qb, qd, qt, qh;
    int remap;   // spatial: 1 = x/q are one row-major image, 0 = four per-direction scans
    int q_mode;  // 0 = raw queries (normalized in P1), 1 = unit-norm fp32 packed queries
    void* y;     // kKindSeq output, dtype of x, packed [B,R,heads,L,D]
    float* out;  // spatial output, fp32 [B,H,W,C]
    int64_t ob;
    const float* skip;
    int skip_per_dir;
    const float* weight;
    int B, R, heads, L, H, W, C;
    int chunk[4];
    int kind, nch, tile;
    SrnlConsts k;
};

// Loops over head_dim are fully unrolled up to D = 16 (every shipped model); larger head
// dims keep the loops rolled so the front end stays fast (they are correctness paths).
template <int D>
struct Unroll {
    static constexpr int v = D <= 16 ? D : 1;
};

template <int D>
struct ScanGeom {
    static constexpr int SROWS = 3 * D + 2;  // m rows [0,D), v rows [D,2D), k rows [2D,3D), e, a
    static constexpr int SP = D + 4;         // padded row stride in floats (16-byte multiple)
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Shared-memory carve-up (identical on host and device).
template <int D, typename XT, typename QT>
struct ScanSmem {
    size_t S, G, K, Dv, EFF, ALP, Y, WS, XB, QB, total;
    __host__ __device__ ScanSmem(int nch, int tile, bool spatial) {
        using Gm = ScanGeom<D>;
        size_t off = 0;
        S = off;   off += align16(sizeof(float) * nch * Gm::SROWS * Gm::SP);
        G = off;   off += align16(sizeof(float) * nch * D * Gm::SP);
        K = off;   off += align16(sizeof(float) * nch * tile * Gm::SP);
        Dv = off;  off += align16(sizeof(float) * nch * tile * Gm::SP);
        EFF = off; off += align16(sizeof(float) * nch * tile);
        ALP = off; off += align16(sizeof(float) * nch * tile);
        Y = off;   off += spatial ? align16(sizeof(float) * nch * tile * Gm::SP) : 0;
        WS = off;  off += align16(sizeof(float) * nch * 2 * D);
        XB = off;  off += align16(sizeof(XT) * 2 * nch * tile * D);
        QB = off;  off += align16(sizeof(QT) * 2 * nch * tile * D);
        total = off;
    }
};

struct ChainInfo {
    int b, dir, head, valid;
    int Lc, nchunks;
};

__device__ __forceinline__ ChainInfo chain_of(const ScanParams& p, int slot) {
    ChainInfo c;
    if (p.kind == kKindSeq) {
        const int idx = blockIdx.x * p.nch + slot;
        c.valid = idx < p.B * p.heads;
        c.b = c.valid ? idx / p.heads : 0;
        c.head = c.valid ? idx % p.heads : 0;
        c.dir = blockIdx.y;
        c.Lc = p.chunk[c.dir];
        c.nchunks = (p.L + c.Lc - 1) / c.Lc;
    } else {
        const int pair = blockIdx.x * (p.nch >> 1) + (slot >> 1);
        c.valid = pair < p.B * p.heads;
        c.b = c.valid ? pair / p.heads : 0;
        c.head = c.valid ? pair % p.heads : 0;
        c.dir = 2 * p.kind + (slot & 1);
        c.Lc = p.kind == kKindRows ? p.W : p.H;
        c.nchunks = p.kind == kKindRows ? p.H : p.W;
    }
    return c;
}

// Pixel (row-major index) that scan `dir` visits at token t (models/operator.py:79-86,
// parallel_line.cuh:16-18).
__device__ __forceinline__ int64_t scan_pixel(int dir, int64_t t, int64_t L, int H, int W) {
    const int64_t orig = (dir & 1) ? L - 1 - t : t;
    return dir < 2 ? orig : (orig % H) * W + orig / H;
}

template <typename T>
__device__ __forceinline__ const T* token_src(const ScanParams& p, const T* base, bool is_q,
                                              const ChainInfo& c, int64_t t) {
    if (p.kind == kKindSeq) {
        const int D = p.C / p.heads;
        if (is_q && p.q_mode == 0)  // raw queries [B,R,L,C]
            return base + (((int64_t)c.b * p.R + c.dir) * p.L + t) * p.C + (int64_t)c.head * D;
        // packed [B,R,heads,L,D]
        return base + (((int64_t)c.b * p.R + c.dir) * p.heads + c.head) * p.L * D + t * D;
    }
    const int64_t sb = is_q ? p.qb : p.xb, sd = is_q ? p.qd : p.xd, st = is_q ? p.qt : p.xt,
                  sh = is_q ? p.qh : p.xh;
    if (p.remap)
        return base + c.b * sb + scan_pixel(c.dir, t, p.L, p.H, p.W) * st + c.head * sh;
    return base + c.b * sb + c.dir * sd + t * st + c.head * sh;
}

// Issue the cp.async copies of one token tile (all chains of the CTA) into buffer `buf`.
template <int D, typename T>
__device__ __forceinline__ void load_tile(const ScanParams& p, const T* base, bool is_q, T* sbuf,
                                          int tile, int c, int j) {
    constexpr int ROWB = D * (int)sizeof(T);
    constexpr int VB = ROWB < 16 ? ROWB : 16;
    constexpr int NV = ROWB / VB;
    const int items = p.nch * tile * NV;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        const int v = it % NV;
        const int tok = (it / NV) % tile;
        const int slot = it / (NV * tile);
        const ChainInfo ch = chain_of(p, slot);
        const int tin = j * tile + tok;
        const int64_t t = (int64_t)c * ch.Lc + tin;
        char* dst = reinterpret_cast<char*>(sbuf + ((size_t)slot * tile + tok) * D) + v * VB;
        if (ch.valid && tin < ch.Lc && t < p.L) {
            const char* src = reinterpret_cast<const char*>(token_src<T>(p, base, is_q, ch, t)) + v * VB;
            cp_async<VB>(dst, src);
        } else {
            // Tail padding and idle slots read as zeros (models/srnl_core/chunk.py:202-206).
            if constexpr (VB == 16) *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
            else if constexpr (VB == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(0, 0);
            else *reinterpret_cast<uint32_t*>(dst) = 0u;
        }
    }
}

__device__ __forceinline__ float softplus_f(float p) { return p > 20.f ? p : log1pf(expf(p)); }

template <int D, typename XT, typename QT, int KIND>
__global__ void __launch_bounds__(kScanThreads) srnl_scan_kernel(const ScanParams p) {
    using Gm = ScanGeom<D>;
    constexpr int SROWS = Gm::SROWS, SP = Gm::SP;
    constexpr bool kSpatial = KIND != kKindSeq;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nch = p.nch, tile = p.tile;
    const ScanSmem<D, XT, QT> lay(nch, tile, kSpatial);
    float* S = reinterpret_cast<float*>(smem_raw + lay.S);
    float* Gs = reinterpret_cast<float*>(smem_raw + lay.G);
    float* Kt = reinterpret_cast<float*>(smem_raw + lay.K);
    float* Dt = reinterpret_cast<float*>(smem_raw + lay.Dv);
    float* EFF = reinterpret_cast<float*>(smem_raw + lay.EFF);
    float* ALP = reinterpret_cast<float*>(smem_raw + lay.ALP);
    float* Yst = reinterpret_cast<float*>(smem_raw + lay.Y);
    float* WS = reinterpret_cast<float*>(smem_raw + lay.WS);
    XT* xbuf = reinterpret_cast<XT*>(smem_raw + lay.XB);
    QT* qbuf = reinterpret_cast<QT*>(smem_raw + lay.QB);
    const XT* xg = static_cast<const XT*>(p.x);
    const QT* qg = static_cast<const QT*>(p.q);
    const int tid = threadIdx.x;

    // ---- load initial memories into the stacked state, and per-slot fusion weights ----
    for (int it = tid; it < nch * SROWS * D; it += blockDim.x) {
        const int col = it % D, row = (it / D) % SROWS, slot = it / (D * SROWS);
        const ChainInfo ch = chain_of(p, slot);
        const int64_t sidx = p.mem_per_chain
                                 ? ((int64_t)ch.b * p.R + ch.dir) * p.heads + ch.head
                                 : (int64_t)ch.dir * p.heads + ch.head;
        float v = 0.f;
        if (ch.valid) {
            if (row < D) v = p.Mm[(sidx * D + row) * D + col];
            else if (row < 2 * D) v = p.Mv[(sidx * D + row - D) * D + col];
            else if (row < 3 * D) v = p.Mk[(sidx * D + row - 2 * D) * D + col];
            else if (row == 3 * D) v = p.Me[sidx * D + col];
            else v = p.Ma[sidx * D + col];
        }
        S[((size_t)slot * SROWS + row) * SP + col] = v;
    }
    if constexpr (kSpatial) {
        for (int it = tid; it < nch * D; it += blockDim.x) {
            const int i = it % D, slot = it / D;
            const ChainInfo ch = chain_of(p, slot);
            const int chn = ch.head * D + i;
            WS[(slot * 2 + 0) * D + i] = ch.valid ? p.weight[ch.dir * p.C + chn] : 0.f;
            WS[(slot * 2 + 1) * D + i] =
                ch.valid ? p.skip[(p.skip_per_dir ? ch.dir * p.C : 0) + chn] : 0.f;
        }
    }

    // Every chain of the CTA shares Lc and the chunk count (the host groups them so).
    const ChainInfo c0 = chain_of(p, 0);
    const int Lc = c0.Lc, nchunks = c0.nchunks;
    const int tiles_per_chunk = (Lc + tile - 1) / tile;
    const int steps = nchunks * tiles_per_chunk;

    // P1 / P2 roles.
    const int p1_slot = tid / tile, p1_tok = tid % tile;
    const bool p1_on = p1_slot < nch;
    const int p2_slot = tid / D, p2_row = tid % D;
    const bool p2_on = p2_slot < nch && chain_of(p, p2_slot).valid;

    // Prefetch step 0.
    load_tile<D, XT>(p, xg, false, xbuf, tile, 0, 0);
    load_tile<D, QT>(p, qg, true, qbuf, tile, 0, 0);
    cp_async_commit();

    float g[D];
    for (int s = 0; s < steps; ++s) {
        const int c = s / tiles_per_chunk, j = s % tiles_per_chunk;
        const int count = min(tile, Lc - j * tile);
        const int buf = s & 1;
        cp_async_wait<0>();
        __syncthreads();  // tile s landed; previous tile's consumers are done
        if (s + 1 < steps) {
            const int cn = (s + 1) / tiles_per_chunk, jn = (s + 1) % tiles_per_chunk;
            const size_t off = (size_t)(buf ^ 1) * nch * tile * D;
            load_tile<D, XT>(p, xg, false, xbuf + off, tile, cn, jn);
            load_tile<D, QT>(p, qg, true, qbuf + off, tile, cn, jn);
        }
        cp_async_commit();
        const XT* xb_cur = xbuf + (size_t)buf * nch * tile * D;
        const QT* qb_cur = qbuf + (size_t)buf * nch * tile * D;

        // ------------------------------- P1 -------------------------------------------
        if (p1_on && p1_tok < count) {
            const ChainInfo ch = chain_of(p, p1_slot);
            const float* Sc = S + (size_t)p1_slot * SROWS * SP;
            const int row = p1_slot * tile + p1_tok;
            const int64_t t = (int64_t)c * Lc + j * tile + p1_tok;
            float qv[D];
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; i += 4) {
                const float4 v4 = load4(qb_cur + (size_t)row * D + i);
                qv[i] = v4.x; qv[i + 1] = v4.y; qv[i + 2] = v4.z; qv[i + 3] = v4.w;
            }
            if (p.q_mode == 0) {
                float qs = 0.f;
#pragma unroll (Unroll<D>::v)
                for (int i = 0; i < D; ++i) qs = fmaf(qv[i], qv[i], qs);
                const float qinv = 1.f / fmaxf(sqrtf(qs), 1e-12f);
#pragma unroll (Unroll<D>::v)
                for (int i = 0; i < D; ++i) qv[i] *= qinv;
            }
            // y = M_m q (output of the chunk-start content memory)
            float yv[D];
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; ++i) {
                float a0 = 0.f, a1 = 0.f;
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4) {
                    const float4 m4 = *reinterpret_cast<const float4*>(Sc + i * SP + jj);
                    a0 = fmaf(m4.x, qv[jj], a0);
                    a1 = fmaf(m4.y, qv[jj + 1], a1);
                    a0 = fmaf(m4.z, qv[jj + 2], a0);
                    a1 = fmaf(m4.w, qv[jj + 3], a1);
                }
                yv[i] = a0 + a1;
            }
            if constexpr (kSpatial) {
#pragma unroll (Unroll<D>::v)
                for (int i = 0; i < D; i += 4)
                    *reinterpret_cast<float4*>(Yst + (size_t)row * SP + i) =
                        make_float4(yv[i], yv[i + 1], yv[i + 2], yv[i + 3]);
            } else {
                if (ch.valid && t < p.L) {
                    XT* yo = static_cast<XT*>(p.y) +
                             (((int64_t)ch.b * p.R + ch.dir) * p.heads + ch.head) * p.L * D + t * D;
#pragma unroll (Unroll<D>::v)
                    for (int i = 0; i < D; i += 4)
                        store4(yo + i, make_float4(yv[i], yv[i + 1], yv[i + 2], yv[i + 3]));
                }
            }
            float xv[D];
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; i += 4) {
                const float4 v4 = load4(xb_cur + (size_t)row * D + i);
                xv[i] = v4.x; xv[i + 1] = v4.y; xv[i + 2] = v4.z; xv[i + 3] = v4.w;
            }
            float kr[D], vv[D];
            float kn = 0.f;
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; ++i) {
                float ak0 = 0.f, ak1 = 0.f, av0 = 0.f, av1 = 0.f;
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(Sc + (2 * D + i) * SP + jj);
                    const float4 v4 = *reinterpret_cast<const float4*>(Sc + (D + i) * SP + jj);
                    ak0 = fmaf(k4.x, xv[jj], ak0);
                    ak1 = fmaf(k4.y, xv[jj + 1], ak1);
                    ak0 = fmaf(k4.z, xv[jj + 2], ak0);
                    ak1 = fmaf(k4.w, xv[jj + 3], ak1);
                    av0 = fmaf(v4.x, xv[jj], av0);
                    av1 = fmaf(v4.y, xv[jj + 1], av1);
                    av0 = fmaf(v4.z, xv[jj + 2], av0);
                    av1 = fmaf(v4.w, xv[jj + 3], av1);
                }
                kr[i] = ak0 + ak1;
                vv[i] = av0 + av1;
                kn = fmaf(kr[i], kr[i], kn);
            }
            const float kinv = 1.f / sqrtf(kn + 1e-6f);
            float ke = 0.f, dn2 = 0.f, ep = 0.f, ap = 0.f;
            const float* ev = Sc + 3 * D * SP;
            const float* avp = Sc + (3 * D + 1) * SP;
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; ++i) {
                const float kk = kr[i] * kinv;
                const float d = kk - vv[i];
                kr[i] = kk;
                vv[i] = d;
                ke = fmaf(kk, kk, ke);
                dn2 = fmaf(d, d, dn2);
                ep = fmaf(xv[i], ev[i], ep);
                ap = fmaf(xv[i], avp[i], ap);
            }
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D; i += 4) {
                *reinterpret_cast<float4*>(Kt + (size_t)row * SP + i) =
                    make_float4(kr[i], kr[i + 1], kr[i + 2], kr[i + 3]);
                *reinterpret_cast<float4*>(Dt + (size_t)row * SP + i) =
                    make_float4(vv[i], vv[i + 1], vv[i + 2], vv[i + 3]);
            }
            ep = fminf(10.f, fmaxf(-10.f, ep));
            ap = fminf(10.f, fmaxf(-10.f, ap + p.k.retention_bias));
            const float eta = p.k.step_scale * softplus_f(ep);
            const float alpha =
                p.k.min_retention + (1.f - p.k.min_retention) * (1.f / (1.f + expf(-ap)));
            const float dn = sqrtf(dn2 + 1e-12f);
            const float cap = p.k.injection_margin * (1.f - alpha) / (dn + 1e-6f);
            float eff = cap * (-expm1f(-(eta / cap)));
            if (p.k.spectral_clamp) {
                const float lim = nextafterf(p.k.spectral_factor * alpha / fmaxf(ke, 1e-20f), 0.f);
                eff = fminf(eff, lim);
            }
            EFF[row] = eff;
            ALP[row] = alpha;
        }
        __syncthreads();

        // ------------------------- fused spatial output ---------------------------------
        if constexpr (kSpatial) {
            constexpr int G4 = D / 4;
            const int items = nch * count * G4;
            for (int it = tid; it < items; it += blockDim.x) {
                const int g4 = it % G4;
                const int tok = (it / G4) % count;
                const int slot = it / (G4 * count);
                const ChainInfo ch = chain_of(p, slot);
                if (!ch.valid) continue;
                const int tin = j * tile + tok;
                const int64_t pix = scan_pixel(ch.dir, (int64_t)c * Lc + tin, p.L, p.H, p.W);
                const int h = (int)(pix / p.W), w = (int)(pix % p.W);
                // Partner direction (same pass) event for this pixel.
                int pc, ptin;
                if (KIND == kKindRows) {
                    const bool even = (ch.dir & 1) == 0;
                    pc = even ? p.H - 1 - h : h;
                    ptin = even ? p.W - 1 - w : w;
                } else {
                    const bool even = (ch.dir & 1) == 0;
                    pc = even ? p.W - 1 - w : w;
                    ptin = even ? p.H - 1 - h : h;
                }
                const int pj = ptin / tile;
                const bool coincident = (pc == c) && (pj == j);
                const bool partner_later = (pc > c) || (pc == c && pj > j);
                if (coincident && (ch.dir & 1)) continue;  // the even direction writes both
                const int i0 = g4 * 4;
                const int row = slot * tile + tok;
                const float4 y4 = *reinterpret_cast<const float4*>(Yst + (size_t)row * SP + i0);
                const float4 x4 = load4(xb_cur + (size_t)row * D + i0);
                const float* wv = WS + (slot * 2) * D + i0;
                const float* sv = WS + (slot * 2 + 1) * D + i0;
                float4 v;
                v.x = wv[0] * (y4.x + sv[0] * x4.x);
                v.y = wv[1] * (y4.y + sv[1] * x4.y);
                v.z = wv[2] * (y4.z + sv[2] * x4.z);
                v.w = wv[3] * (y4.w + sv[3] * x4.w);
                float* o = p.out + (int64_t)ch.b * p.ob + pix * p.C + ch.head * D + i0;
                if (coincident) {
                    const int pslot = slot ^ 1;
                    const int prow = pslot * tile + (ptin - j * tile);
                    const float4 py = *reinterpret_cast<const float4*>(Yst + (size_t)prow * SP + i0);
                    const float4 px = load4(xb_cur + (size_t)prow * D + i0);
                    const float* pw = WS + (pslot * 2) * D + i0;
                    const float* ps = WS + (pslot * 2 + 1) * D + i0;
                    float4 u;
                    u.x = pw[0] * (py.x + ps[0] * px.x);
                    u.y = pw[1] * (py.y + ps[1] * px.y);
                    u.z = pw[2] * (py.z + ps[2] * px.z);
                    u.w = pw[3] * (py.w + ps[3] * px.w);
                    if (KIND == kKindRows) {
                        v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
                    } else {
                        const float4 prev = *reinterpret_cast<const float4*>(o);
                        v.x = (prev.x + v.x) + u.x;
                        v.y = (prev.y + v.y) + u.y;
                        v.z = (prev.z + v.z) + u.z;
                        v.w = (prev.w + v.w) + u.w;
                    }
                } else if (KIND == kKindCols || !partner_later) {
                    const float4 prev = *reinterpret_cast<const float4*>(o);
                    v.x += prev.x; v.y += prev.y; v.z += prev.z; v.w += prev.w;
                }
                *reinterpret_cast<float4*>(o) = v;
            }
        }

        // ------------------------------- P2 -------------------------------------------
        if (p2_on) {
            if (j == 0) {
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; ++jj) g[jj] = jj == p2_row ? 1.f : 0.f;
            }
            const int base = p2_slot * tile;
            for (int t = 0; t < count; ++t) {
                const float* kt = Kt + (size_t)(base + t) * SP;
                const float di = Dt[(size_t)(base + t) * SP + p2_row];
                const float a = ALP[base + t], e = EFF[base + t];
                float r0 = di, r1 = 0.f, r2 = 0.f, r3 = 0.f;
                float kv[D];
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kt + jj);
                    kv[jj] = k4.x; kv[jj + 1] = k4.y; kv[jj + 2] = k4.z; kv[jj + 3] = k4.w;
                    r0 = fmaf(g[jj], k4.x, r0);
                    r1 = fmaf(g[jj + 1], k4.y, r1);
                    r2 = fmaf(g[jj + 2], k4.z, r2);
                    r3 = fmaf(g[jj + 3], k4.w, r3);
                }
                const float u = e * ((r0 + r1) + (r2 + r3));
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; ++jj) g[jj] = fmaf(-u, kv[jj], a * g[jj]);
            }
            if (j == tiles_per_chunk - 1) {
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4)
                    *reinterpret_cast<float4*>(Gs + ((size_t)p2_slot * D + p2_row) * SP + jj) =
                        make_float4(g[jj], g[jj + 1], g[jj + 2], g[jj + 3]);
            }
        }
        if (j == tiles_per_chunk - 1) {
            __syncthreads();
            // ------------------------------- P3 ---------------------------------------
            if (c + 1 < nchunks) {
                for (int task = tid; task < nch * SROWS; task += blockDim.x) {
                    const int slot = task / SROWS;
                    if (!chain_of(p, slot).valid) continue;
                    float* rowp = S + (size_t)task * SP;
                    const float* Gc = Gs + (size_t)slot * D * SP;
                    float rv[D], acc[D];
#pragma unroll (Unroll<D>::v)
                    for (int jj = 0; jj < D; jj += 4) {
                        const float4 r4 = *reinterpret_cast<const float4*>(rowp + jj);
                        rv[jj] = r4.x; rv[jj + 1] = r4.y; rv[jj + 2] = r4.z; rv[jj + 3] = r4.w;
                    }
#pragma unroll (Unroll<D>::v)
                    for (int jj = 0; jj < D; ++jj) acc[jj] = 0.f;
#pragma unroll (Unroll<D>::v)
                    for (int l = 0; l < D; ++l) {
#pragma unroll (Unroll<D>::v)
                        for (int jj = 0; jj < D; jj += 4) {
                            const float4 g4v = *reinterpret_cast<const float4*>(Gc + l * SP + jj);
                            acc[jj] = fmaf(rv[l], g4v.x, acc[jj]);
                            acc[jj + 1] = fmaf(rv[l], g4v.y, acc[jj + 1]);
                            acc[jj + 2] = fmaf(rv[l], g4v.z, acc[jj + 2]);
                            acc[jj + 3] = fmaf(rv[l], g4v.w, acc[jj + 3]);
                        }
                    }
#pragma unroll (Unroll<D>::v)
                    for (int jj = 0; jj < D; jj += 4)
                        *reinterpret_cast<float4*>(rowp + jj) =
                            make_float4(acc[jj], acc[jj + 1], acc[jj + 2], acc[jj + 3]);
                }
            }
        }
    }
    cp_async_wait<0>();
}

}  // namespace vh
