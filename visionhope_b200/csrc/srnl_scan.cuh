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
// Chunks longer than the token tile are processed tile by tile with G carried in registers.
// Each P1 thread keeps the same (chain, token slot) for the whole scan and prefetches its
// next token's x and q into registers one step ahead.
//
// Kinds:
//   kKindRows / kKindCols: the fused spatial operator (fused.cu:307-351 +
//      parallel_line.cuh:2-59).  A CTA holds (b, head) pairs of scans {0,1} (rows pass) or
//      {2,3} (columns pass); each token thread writes weight_d * (y_d + skip_d x_d) straight
//      to the fp32 output.  The rows pass runs first.  Within a pass every pixel is touched
//      exactly twice, by the two scans of the pair, and which touch comes first is a fixed
//      function of (chunk, tile): the first touch of the rows pass stores, every other touch
//      adds, and two touches in the same step (the middle row/column of an odd image) are
//      ordered by a barrier.  The result is deterministic and needs no atomics, no
//      per-direction planes and no merge kernel.
//   kKindSeq: packed sequences (fused.cu:93-179, chunk.cu:252-509, lines.cu:3-237), y out.
#pragma once

#include <type_traits>

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
    int kind, nch, tile, log2tile;
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
template <int D>
struct ScanSmem {
    size_t S, G, K, Dv, EFF, ALP, WS, total;
    __host__ __device__ ScanSmem(int nch, int tile) {
        using Gm = ScanGeom<D>;
        size_t off = 0;
        S = off;   off += align16(sizeof(float) * nch * Gm::SROWS * Gm::SP);
        G = off;   off += align16(sizeof(float) * nch * D * Gm::SP);
        K = off;   off += align16(sizeof(float) * nch * tile * Gm::SP);
        Dv = off;  off += align16(sizeof(float) * nch * tile * Gm::SP);
        EFF = off; off += align16(sizeof(float) * nch * tile);
        ALP = off; off += align16(sizeof(float) * nch * tile);
        WS = off;  off += align16(sizeof(float) * nch * 2 * D);
        total = off;
    }
};

struct Chain {
    int b, dir, head, valid;
};

__device__ __forceinline__ Chain chain_of(const ScanParams& p, int slot) {
    Chain c;
    int idx;
    if (p.kind == kKindSeq) {
        idx = blockIdx.x * p.nch + slot;
        c.dir = blockIdx.y;
    } else {
        idx = blockIdx.x * (p.nch >> 1) + (slot >> 1);
        c.dir = 2 * p.kind + (slot & 1);
    }
    c.valid = idx < p.B * p.heads;
    c.b = c.valid ? idx / p.heads : 0;
    c.head = c.valid ? idx % p.heads : 0;
    return c;
}

// Pixel (row-major) that scan `dir` visits at token `tin` of chunk `c`: rows are the chunks
// of scans 0/1, columns those of scans 2/3; odd scans run backwards (models/operator.py:79-86,
// parallel_line.cuh:16-18).  No division: the chunk index is the row/column index.
__device__ __forceinline__ int scan_pixel(int dir, int c, int tin, int H, int W) {
    switch (dir) {
        case 0: return c * W + tin;
        case 1: return (H - 1 - c) * W + (W - 1 - tin);
        case 2: return tin * W + c;
        default: return (H - 1 - tin) * W + (W - 1 - c);
    }
}

// One token's D elements held raw in registers (vector loads of up to 16 bytes).
template <int D, typename T>
struct RowReg {
    static constexpr int BYTES = D * (int)sizeof(T);
    static constexpr int VB = BYTES >= 16 ? 16 : BYTES;
    static constexpr int NV = BYTES / VB;
    using V = typename std::conditional<VB == 16, uint4,
                                        typename std::conditional<VB == 8, uint2, uint32_t>::type>::type;
    V v[NV];
    __device__ __forceinline__ void load(const T* p) {
        const V* s = reinterpret_cast<const V*>(p);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = __ldg(s + i);
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = V{};
    }
    __device__ __forceinline__ void to_float(float* f) const {
        const T* e = reinterpret_cast<const T*>(v);
#pragma unroll (Unroll<D>::v)
        for (int i = 0; i < D; i += 4) {
            const float4 t = load4(e + i);
            f[i] = t.x; f[i + 1] = t.y; f[i + 2] = t.z; f[i + 3] = t.w;
        }
    }
};

__device__ __forceinline__ float softplus_f(float p) { return p > 20.f ? p : log1pf(expf(p)); }

template <int D, typename XT, typename QT, int KIND>
__global__ void __launch_bounds__(kScanThreads, 4) srnl_scan_kernel(const ScanParams p) {
    using Gm = ScanGeom<D>;
    constexpr int SROWS = Gm::SROWS, SP = Gm::SP;
    constexpr bool kSpatial = KIND != kKindSeq;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nch = p.nch, tile = p.tile, lt = p.log2tile;
    const ScanSmem<D> lay(nch, tile);
    float* S = reinterpret_cast<float*>(smem_raw + lay.S);
    float* Gs = reinterpret_cast<float*>(smem_raw + lay.G);
    float* Kt = reinterpret_cast<float*>(smem_raw + lay.K);
    float* Dt = reinterpret_cast<float*>(smem_raw + lay.Dv);
    float* EFF = reinterpret_cast<float*>(smem_raw + lay.EFF);
    float* ALP = reinterpret_cast<float*>(smem_raw + lay.ALP);
    float* WS = reinterpret_cast<float*>(smem_raw + lay.WS);
    const int tid = threadIdx.x;

    // ---- initial memories -> stacked state; per-slot fusion weights ---------------------
    for (int slot = 0; slot < nch; ++slot) {
        const Chain ch = chain_of(p, slot);
        const int64_t sidx = p.mem_per_chain ? ((int64_t)ch.b * p.R + ch.dir) * p.heads + ch.head
                                             : (int64_t)ch.dir * p.heads + ch.head;
        float* Sc = S + (size_t)slot * SROWS * SP;
        for (int it = tid; it < SROWS * D; it += blockDim.x) {
            const int col = it % D, row = it / D;
            float v = 0.f;
            if (ch.valid) {
                if (row < D) v = p.Mm[(sidx * D + row) * D + col];
                else if (row < 2 * D) v = p.Mv[(sidx * D + row - D) * D + col];
                else if (row < 3 * D) v = p.Mk[(sidx * D + row - 2 * D) * D + col];
                else if (row == 3 * D) v = p.Me[sidx * D + col];
                else v = p.Ma[sidx * D + col];
            }
            Sc[row * SP + col] = v;
        }
        if constexpr (kSpatial) {
            for (int i = tid; i < D; i += blockDim.x) {
                const int chn = ch.head * D + i;
                WS[(slot * 2 + 0) * D + i] = ch.valid ? p.weight[ch.dir * p.C + chn] : 0.f;
                WS[(slot * 2 + 1) * D + i] =
                    ch.valid ? p.skip[(p.skip_per_dir ? ch.dir * p.C : 0) + chn] : 0.f;
            }
        }
    }

    // ---- geometry shared by every chain of the CTA -------------------------------------
    int Lc, nchunks;
    if (KIND == kKindRows) {
        Lc = p.W;
        nchunks = p.H;
    } else if (KIND == kKindCols) {
        Lc = p.H;
        nchunks = p.W;
    } else {
        Lc = p.chunk[blockIdx.y];
        nchunks = (p.L + Lc - 1) / Lc;
    }
    const int tpc = (Lc + tile - 1) >> lt;  // tiles per chunk

    // ---- P1 role: one (chain, token slot) per thread ------------------------------------
    const int p1_slot = tid >> lt, p1_tok = tid & (tile - 1);
    const Chain c1 = chain_of(p, p1_slot < nch ? p1_slot : 0);
    const bool p1_on = p1_slot < nch && c1.valid;
    const XT* xbase;
    const QT* qbase;
    int64_t xts, qts;
    float* obase = nullptr;
    XT* ybase = nullptr;
    if constexpr (kSpatial) {
        xbase = static_cast<const XT*>(p.x) + c1.b * p.xb + c1.head * p.xh + (p.remap ? 0 : c1.dir * p.xd);
        qbase = static_cast<const QT*>(p.q) + c1.b * p.qb + c1.head * p.qh + (p.remap ? 0 : c1.dir * p.qd);
        xts = p.xt;
        qts = p.qt;
        obase = p.out + c1.b * p.ob + c1.head * D;
    } else {
        const int64_t chain = ((int64_t)c1.b * p.R + c1.dir) * p.heads + c1.head;
        xbase = static_cast<const XT*>(p.x) + chain * p.L * D;
        xts = D;
        if (p.q_mode == 0) {
            qbase = static_cast<const QT*>(p.q) + ((int64_t)c1.b * p.R + c1.dir) * p.L * p.C + c1.head * D;
            qts = p.C;
        } else {
            qbase = static_cast<const QT*>(p.q) + chain * p.L * D;
            qts = D;
        }
        ybase = static_cast<XT*>(p.y) + chain * p.L * D;
    }

    // ---- P2 role: one row of one chain's G per thread -----------------------------------
    const int p2_slot = tid / D, p2_row = tid % D;
    const bool p2_on = p2_slot < nch && chain_of(p, p2_slot).valid;

    RowReg<D, XT> xn;
    RowReg<D, QT> qn;
    auto prefetch = [&](int c, int j) {
        const int tin = (j << lt) + p1_tok;
        const int64_t t = (int64_t)c * Lc + tin;
        if (p1_on && tin < Lc && t < p.L) {
            const int64_t s = (kSpatial && p.remap) ? (int64_t)scan_pixel(c1.dir, c, tin, p.H, p.W) : t;
            xn.load(xbase + s * xts);
            qn.load(qbase + s * qts);
        } else {
            xn.zero();  // tail padding reads as zeros (models/srnl_core/chunk.py:202-206)
            qn.zero();
        }
    };
    prefetch(0, 0);

    float g[D];
    int c = 0, j = 0;
    for (int s = 0, steps = nchunks * tpc; s < steps; ++s) {
        const RowReg<D, XT> xc = xn;
        const RowReg<D, QT> qc = qn;
        const int count = min(tile, Lc - (j << lt));
        const int cn = j + 1 < tpc ? c : c + 1, jn = j + 1 < tpc ? j + 1 : 0;
        __syncthreads();  // P2/P3 of the previous step are done with Kt, Dt, S
        if (s + 1 < steps) prefetch(cn, jn);

        // ------------------------------- P1 -------------------------------------------
        bool deferred = false;
        float4 dv[D / 4];
        float* dptr = nullptr;
        if (p1_on && p1_tok < count) {
            const float* Sc = S + (size_t)p1_slot * SROWS * SP;
            const int row = (p1_slot << lt) + p1_tok;
            const int tin = (j << lt) + p1_tok;
            const int64_t t = (int64_t)c * Lc + tin;
            float qv[D], xv[D];
            qc.to_float(qv);
            xc.to_float(xv);
            if (p.q_mode == 0) {
                float qs = 0.f;
#pragma unroll (Unroll<D>::v)
                for (int i = 0; i < D; ++i) qs = fmaf(qv[i], qv[i], qs);
                const float qinv = 1.f / fmaxf(sqrtf(qs), 1e-12f);
#pragma unroll (Unroll<D>::v)
                for (int i = 0; i < D; ++i) qv[i] *= qinv;
            }
            // y = M_m q from the chunk-start content memory, emitted immediately.
#pragma unroll (Unroll<D>::v)
            for (int i0 = 0; i0 < D; i0 += 4) {
                float yv[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    float a0 = 0.f, a1 = 0.f;
#pragma unroll (Unroll<D>::v)
                    for (int jj = 0; jj < D; jj += 4) {
                        const float4 m4 = *reinterpret_cast<const float4*>(Sc + (i0 + r) * SP + jj);
                        a0 = fmaf(m4.x, qv[jj], a0);
                        a1 = fmaf(m4.y, qv[jj + 1], a1);
                        a0 = fmaf(m4.z, qv[jj + 2], a0);
                        a1 = fmaf(m4.w, qv[jj + 3], a1);
                    }
                    yv[r] = a0 + a1;
                }
                if constexpr (kSpatial) {
                    const float4 w4 = *reinterpret_cast<const float4*>(WS + (p1_slot * 2) * D + i0);
                    const float4 s4 = *reinterpret_cast<const float4*>(WS + (p1_slot * 2 + 1) * D + i0);
                    dv[i0 / 4] = make_float4(w4.x * (yv[0] + s4.x * xv[i0]), w4.y * (yv[1] + s4.y * xv[i0 + 1]),
                                             w4.z * (yv[2] + s4.z * xv[i0 + 2]), w4.w * (yv[3] + s4.w * xv[i0 + 3]));
                } else {
                    if (t < p.L) store4(ybase + t * D + i0, make_float4(yv[0], yv[1], yv[2], yv[3]));
                }
            }
            if constexpr (kSpatial) {
                // The partner scan of the pair visits this pixel at chunk nchunks-1-c, token Lc-1-tin.
                const int pc = nchunks - 1 - c, ptin = Lc - 1 - tin, pj = ptin >> lt;
                const bool coincident = pc == c && pj == j;
                const bool partner_later = pc > c || (pc == c && pj > j);
                const bool even = (c1.dir & 1) == 0;
                dptr = obase + (int64_t)scan_pixel(c1.dir, c, tin, p.H, p.W) * p.C;
                if (coincident && !even) {
                    deferred = true;  // written after the barrier, on top of the even scan's value
                } else {
                    const bool store_only = KIND == kKindRows && (coincident || partner_later);
#pragma unroll (Unroll<D>::v)
                    for (int i = 0; i < D / 4; ++i) {
                        float4 v = dv[i];
                        if (!store_only) {
                            const float4 o = *reinterpret_cast<const float4*>(dptr + 4 * i);
                            v.x = o.x + v.x; v.y = o.y + v.y; v.z = o.z + v.z; v.w = o.w + v.w;
                        }
                        *reinterpret_cast<float4*>(dptr + 4 * i) = v;
                    }
                }
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
                *reinterpret_cast<float4*>(Kt + (size_t)row * SP + i) = make_float4(kr[i], kr[i + 1], kr[i + 2], kr[i + 3]);
                *reinterpret_cast<float4*>(Dt + (size_t)row * SP + i) = make_float4(vv[i], vv[i + 1], vv[i + 2], vv[i + 3]);
            }
            ep = fminf(10.f, fmaxf(-10.f, ep));
            ap = fminf(10.f, fmaxf(-10.f, ap + p.k.retention_bias));
            const float eta = p.k.step_scale * softplus_f(ep);
            const float alpha = p.k.min_retention + (1.f - p.k.min_retention) * (1.f / (1.f + expf(-ap)));
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
        if (kSpatial && deferred) {
#pragma unroll (Unroll<D>::v)
            for (int i = 0; i < D / 4; ++i) {
                const float4 o = *reinterpret_cast<const float4*>(dptr + 4 * i);
                *reinterpret_cast<float4*>(dptr + 4 * i) =
                    make_float4(o.x + dv[i].x, o.y + dv[i].y, o.z + dv[i].z, o.w + dv[i].w);
            }
        }

        // ------------------------------- P2 -------------------------------------------
        if (p2_on) {
            if (j == 0) {
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; ++jj) g[jj] = jj == p2_row ? 1.f : 0.f;
            }
            const int base = p2_slot << lt;
            float4 kq[D / 4];
#pragma unroll (Unroll<D>::v)
            for (int jj = 0; jj < D / 4; ++jj) kq[jj] = *reinterpret_cast<const float4*>(Kt + (size_t)base * SP + 4 * jj);
            float di = Dt[(size_t)base * SP + p2_row];
            float a = ALP[base], e = EFF[base];
            for (int t = 0; t < count; ++t) {
                float kv[D];
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D / 4; ++jj) {
                    kv[4 * jj] = kq[jj].x;
                    kv[4 * jj + 1] = kq[jj].y;
                    kv[4 * jj + 2] = kq[jj].z;
                    kv[4 * jj + 3] = kq[jj].w;
                }
                const float dcur = di, acur = a, ecur = e;
                if (t + 1 < count) {  // prefetch the next token's key and gates
                    const size_t nrow = (size_t)(base + t + 1);
#pragma unroll (Unroll<D>::v)
                    for (int jj = 0; jj < D / 4; ++jj) kq[jj] = *reinterpret_cast<const float4*>(Kt + nrow * SP + 4 * jj);
                    di = Dt[nrow * SP + p2_row];
                    a = ALP[nrow];
                    e = EFF[nrow];
                }
                float r0 = dcur, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4) {
                    r0 = fmaf(g[jj], kv[jj], r0);
                    r1 = fmaf(g[jj + 1], kv[jj + 1], r1);
                    r2 = fmaf(g[jj + 2], kv[jj + 2], r2);
                    r3 = fmaf(g[jj + 3], kv[jj + 3], r3);
                }
                const float u = ecur * ((r0 + r1) + (r2 + r3));
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; ++jj) g[jj] = fmaf(-u, kv[jj], acur * g[jj]);
            }
            if (j == tpc - 1) {
#pragma unroll (Unroll<D>::v)
                for (int jj = 0; jj < D; jj += 4)
                    *reinterpret_cast<float4*>(Gs + ((size_t)p2_slot * D + p2_row) * SP + jj) =
                        make_float4(g[jj], g[jj + 1], g[jj + 2], g[jj + 3]);
            }
        }
        if (j == tpc - 1) {
            if (c + 1 < nchunks) {
                __syncthreads();
                // ------------------------------- P3 -----------------------------------
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
                        *reinterpret_cast<float4*>(rowp + jj) = make_float4(acc[jj], acc[jj + 1], acc[jj + 2], acc[jj + 3]);
                }
            }
            ++c;
            j = 0;
        } else {
            ++j;
        }
    }
}

}  // namespace vh
