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
// kKindBoth: rows and columns passes in one launch (warp-per-chain scan only), the columns
// pass accumulating in a second fp32 plane that each CTA folds in at its end.
enum ScanKind { kKindRows = 0, kKindCols = 1, kKindSeq = 2, kKindBoth = 3 };

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
    // spatial, optional: second accumulation plane (out's layout), final cast target and the
    // addend folded in before the cast (io dtype, [B, H, W, C]).
    float* aux;
    const void* addend;
    int64_t ab;
    void* fin;
    int fin_dtype;
    int64_t fb;
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
// Number of bf16 parts the tensor-core path splits each fp32 memory row into (hi + mid + lo
// carry 24 mantissa bits, i.e. fp32-level projections from bf16 x/q operands).
constexpr int kSplits = 3;

template <int D>
struct ScanSmem {
    size_t S, G, K, Dv, EFF, ALP, WS, XS, QS, MB, total;
    __host__ __device__ ScanSmem(int nch, int tile, bool mma = false) {
        using Gm = ScanGeom<D>;
        size_t off = 0;
        S = off;   off += align16(sizeof(float) * nch * Gm::SROWS * Gm::SP);
        G = off;   off += align16(sizeof(float) * nch * D * Gm::SP);
        K = off;   off += align16(sizeof(float) * nch * tile * Gm::SP);
        Dv = off;  off += align16(sizeof(float) * nch * tile * Gm::SP);
        EFF = off; off += align16(sizeof(float) * nch * tile);
        ALP = off; off += align16(sizeof(float) * nch * tile);
        WS = off;  off += align16(sizeof(float) * nch * 2 * D);
        // tensor-core path: bf16 x/q tiles (32-byte rows) and split memories [nch][3][3D rows]
        XS = off;  off += mma ? align16(2 * D * nch * tile) : 0;
        QS = off;  off += mma ? align16(2 * D * nch * tile) : 0;
        MB = off;  off += mma ? align16(2 * D * nch * kSplits * 3 * D) : 0;
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

// The per-token gate arithmetic of every scan.  The reference builds its recurrence kernels
// with --use_fast_math (models/srnl_core/fused.py:78, chunk.py:121), so the exponentials,
// the logarithm, the divisions and the square roots use the approximate hardware forms here
// too; expm1f and the clamp's nextafterf stay exact.

// 1 / sqrt(||k~||^2 + 1e-6), the key normalization (inference_recurrence.cuh:60-66).
__device__ __forceinline__ float key_inv_norm(float kn2) { return rsqrtf(kn2 + 1e-6f); }

// (eta_eff, alpha) of one token from x.e and x.a (before clamping), ke = ||k||^2 of the
// normalized key and dn2 = ||k - v||^2: eta = step_scale softplus(x.e) (softplus as the
// reference writes it, log(1 + exp(p)), inference_recurrence.cuh:74), alpha = min_ret +
// (1 - min_ret) sigmoid(x.a + bias), the injection cap and the spectral clamp
// (inference_recurrence.cuh:66-90, memory.cuh:219-233).
__device__ __forceinline__ float2 token_gate_scalars(const SrnlConsts& K, float xe, float xa, float ke, float dn2) {
    const float ep = fminf(10.f, fmaxf(-10.f, xe));
    const float ap = fminf(10.f, fmaxf(-10.f, xa + K.retention_bias));
    const float eta = K.step_scale * (ep > 20.f ? ep : __logf(1.f + __expf(ep)));
    const float alpha = K.min_retention + (1.f - K.min_retention) * __fdividef(1.f, 1.f + __expf(-ap));
    const float dsq = dn2 + 1e-12f;
    const float dn = dsq * rsqrtf(dsq);
    const float cap = __fdividef(K.injection_margin * (1.f - alpha), dn + 1e-6f);
    float eff = cap * (-expm1f(-__fdividef(eta, cap)));
    if (K.spectral_clamp) {
        const float lim = nextafterf(__fdividef(K.spectral_factor * alpha, fmaxf(ke, 1e-20f)), 0.f);
        eff = fminf(eff, lim);
    }
    return make_float2(eff, alpha);
}

// ---- tensor-core helpers (bf16 m16n8k16, fp32 accumulate) ------------------------------
// Rows of 16 bf16 (32 bytes) are stored with their two 16-byte halves swapped on rows whose
// bit 2 is set, so each 8-row ldmatrix phase touches 8 distinct bank groups.
__device__ __forceinline__ int swz(int row, int half) { return row * 32 + ((half ^ ((row >> 2) & 1)) << 4); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const unsigned char* p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// Writes the three bf16 parts of one 16-value fp32 memory row (row `r` of the stacked state)
// into the split-memory block of a chain: part k = bf16(v - sum of earlier parts).
__device__ __forceinline__ void write_splits16(unsigned char* mb_slot, int r, const float* v) {
    float rem[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) rem[i] = v[i];
#pragma unroll
    for (int k = 0; k < kSplits; ++k) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(rem[2 * i], rem[2 * i + 1]);
            const float2 hf = __bfloat1622float2(h);
            rem[2 * i] -= hf.x;
            rem[2 * i + 1] -= hf.y;
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        unsigned char* base = mb_slot + k * 48 * 32;
        *reinterpret_cast<uint4*>(base + swz(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(base + swz(r, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// MMA selects the tensor-core token phase (D = 16, bf16 x and raw bf16 q, tile >= 16): the
// projections k~ = M_k x, v = M_v x and M_m q_raw run as bf16 m16n8k16 MMAs against a three-way
// bf16 split of the fp32 memories (fp32 accumulate), and y is scaled by 1/||q_raw|| afterwards.
template <int D, typename XT, typename QT, int KIND, bool MMA = false>
__global__ void __launch_bounds__(kScanThreads, 4) srnl_scan_kernel(const ScanParams p) {
    using Gm = ScanGeom<D>;
    constexpr int SROWS = Gm::SROWS, SP = Gm::SP;
    constexpr bool kSpatial = KIND != kKindSeq;
    static_assert(!MMA || (D == 16 && std::is_same<XT, __nv_bfloat16>::value &&
                           std::is_same<QT, __nv_bfloat16>::value),
                  "the tensor-core token phase is specialised for D = 16 bf16 inputs");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int nch = p.nch, tile = p.tile, lt = p.log2tile;
    const ScanSmem<D> lay(nch, tile, MMA);
    float* S = reinterpret_cast<float*>(smem_raw + lay.S);
    float* Gs = reinterpret_cast<float*>(smem_raw + lay.G);
    float* Kt = reinterpret_cast<float*>(smem_raw + lay.K);
    float* Dt = reinterpret_cast<float*>(smem_raw + lay.Dv);
    float* EFF = reinterpret_cast<float*>(smem_raw + lay.EFF);
    float* ALP = reinterpret_cast<float*>(smem_raw + lay.ALP);
    float* WS = reinterpret_cast<float*>(smem_raw + lay.WS);
    unsigned char* Xs = smem_raw + lay.XS;
    unsigned char* Qs = smem_raw + lay.QS;
    unsigned char* Mb = smem_raw + lay.MB;
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

    if constexpr (MMA) {
        __syncthreads();  // the stacked state is complete
        for (int task = tid; task < nch * 3 * D; task += blockDim.x) {
            const int slot = task / (3 * D), r = task % (3 * D);
            float v[16];
            const float* rowp = S + ((size_t)slot * SROWS + r) * SP;
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                const float4 f = *reinterpret_cast<const float4*>(rowp + i);
                v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
            }
            write_splits16(Mb + (size_t)slot * kSplits * 48 * 32, r, v);
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

    // ---- tensor-core role: warp w owns CTA rows 32w..32w+31 (two 16-row M-tiles) --------
    const int lane = tid & 31, wrp = tid >> 5, qg = lane >> 2, qt4 = lane & 3;
    int mt_slot[2];
    bool mt_on[2];
    Chain mt_ch[2];
    float* mt_out[2] = {nullptr, nullptr};
    XT* mt_y[2] = {nullptr, nullptr};
    if constexpr (MMA) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            const int rbase = wrp * 32 + mt * 16;
            mt_slot[mt] = rbase >> lt;
            mt_ch[mt] = chain_of(p, mt_slot[mt] < nch ? mt_slot[mt] : 0);
            mt_on[mt] = rbase < nch * tile && mt_ch[mt].valid;
            if (kSpatial) {
                mt_out[mt] = p.out + mt_ch[mt].b * p.ob + mt_ch[mt].head * D;
            } else {
                const int64_t chain = ((int64_t)mt_ch[mt].b * p.R + mt_ch[mt].dir) * p.heads + mt_ch[mt].head;
                mt_y[mt] = static_cast<XT*>(p.y) + chain * p.L * D;
            }
        }
    }

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
        unsigned mdef = 0;  // bit (2 mt + h): this thread defers a middle-row write
        if constexpr (MMA) {
            // Stage this thread's token row (raw bf16) for the warp's ldmatrix loads.
            if (p1_slot < nch) {
                *reinterpret_cast<uint4*>(Xs + swz(tid, 0)) = *reinterpret_cast<const uint4*>(&xc.v[0]);
                *reinterpret_cast<uint4*>(Xs + swz(tid, 1)) = *reinterpret_cast<const uint4*>(&xc.v[1]);
                *reinterpret_cast<uint4*>(Qs + swz(tid, 0)) = *reinterpret_cast<const uint4*>(&qc.v[0]);
                *reinterpret_cast<uint4*>(Qs + swz(tid, 1)) = *reinterpret_cast<const uint4*>(&qc.v[1]);
            }
            __syncwarp();
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                if (!mt_on[mt]) continue;  // warp-uniform
                const int rbase = wrp * 32 + mt * 16, slot = mt_slot[mt];
                uint32_t ax[4], aq[4];
                ldsm_x4(ax, Xs + swz(rbase + (lane & 15), lane >> 4));
                ldsm_x4(aq, Qs + swz(rbase + (lane & 15), lane >> 4));
                float ck[2][4] = {}, cv[2][4] = {}, cy[2][4] = {};
                const unsigned char* mbs = Mb + (size_t)slot * kSplits * 48 * 32;
                const int brow = (lane & 7) + ((lane >> 4) << 3), bhalf = (lane >> 3) & 1;
#pragma unroll
                for (int k = 0; k < kSplits; ++k) {
                    const unsigned char* mb = mbs + k * 48 * 32;
                    uint32_t bm[4], bv[4], bk[4];
                    ldsm_x4(bm, mb + swz(brow, bhalf));            // M_m rows 0-15
                    ldsm_x4(bv, mb + swz(16 + brow, bhalf));       // M_v rows 16-31
                    ldsm_x4(bk, mb + swz(32 + brow, bhalf));       // M_k rows 32-47
                    mma_16816(cy[0], aq, bm[0], bm[1]);
                    mma_16816(cy[1], aq, bm[2], bm[3]);
                    mma_16816(cv[0], ax, bv[0], bv[1]);
                    mma_16816(cv[1], ax, bv[2], bv[3]);
                    mma_16816(ck[0], ax, bk[0], bk[1]);
                    mma_16816(ck[1], ax, bk[2], bk[3]);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // Thread (qg, qt4) holds channels {2t, 2t+1, 8+2t, 9+2t} of token row qg + 8h.
                    const int row = rbase + qg + 8 * h;
                    const int tok = row & (tile - 1);
                    const int tin = (j << lt) + tok;
                    const int64_t t = (int64_t)c * Lc + tin;
                    // Raw k~ and v go to this row's staging slots; the token's own thread
                    // finishes norms and gates below (in-thread, no shuffles).
                    float* krow = Kt + (size_t)row * SP + 2 * qt4;
                    float* drow = Dt + (size_t)row * SP + 2 * qt4;
                    *reinterpret_cast<float2*>(krow) = make_float2(ck[0][2 * h], ck[0][2 * h + 1]);
                    *reinterpret_cast<float2*>(krow + 8) = make_float2(ck[1][2 * h], ck[1][2 * h + 1]);
                    *reinterpret_cast<float2*>(drow) = make_float2(cv[0][2 * h], cv[0][2 * h + 1]);
                    *reinterpret_cast<float2*>(drow + 8) = make_float2(cv[1][2 * h], cv[1][2 * h + 1]);
                    const float2 q01 = bf2_to_f2(aq[h]), q23 = bf2_to_f2(aq[2 + h]);
                    float qs = q01.x * q01.x + q01.y * q01.y + q23.x * q23.x + q23.y * q23.y;
                    qs = quad_sum(qs);
                    if (tok >= count) continue;
                    const float qinv = 1.f / fmaxf(sqrtf(qs), 1e-12f);
                    const float yv[4] = {cy[0][2 * h] * qinv, cy[0][2 * h + 1] * qinv,
                                         cy[1][2 * h] * qinv, cy[1][2 * h + 1] * qinv};
                    if constexpr (kSpatial) {
                        const float2 x01 = bf2_to_f2(ax[h]), x23 = bf2_to_f2(ax[2 + h]);
                        const float* wv = WS + (slot * 2) * D;
                        const float* sv = WS + (slot * 2 + 1) * D;
                        const float2 w_lo = *reinterpret_cast<const float2*>(wv + 2 * qt4);
                        const float2 w_hi = *reinterpret_cast<const float2*>(wv + 8 + 2 * qt4);
                        const float2 s_lo = *reinterpret_cast<const float2*>(sv + 2 * qt4);
                        const float2 s_hi = *reinterpret_cast<const float2*>(sv + 8 + 2 * qt4);
                        const float2 o_lo = make_float2(w_lo.x * (yv[0] + s_lo.x * x01.x), w_lo.y * (yv[1] + s_lo.y * x01.y));
                        const float2 o_hi = make_float2(w_hi.x * (yv[2] + s_hi.x * x23.x), w_hi.y * (yv[3] + s_hi.y * x23.y));
                        const int dir = mt_ch[mt].dir;
                        const int pc = nchunks - 1 - c, ptin = Lc - 1 - tin, pj = ptin >> lt;
                        const bool coincident = pc == c && pj == j;
                        const bool partner_later = pc > c || (pc == c && pj > j);
                        float* op = mt_out[mt] + (int64_t)scan_pixel(dir, c, tin, p.H, p.W) * p.C + 2 * qt4;
                        if (coincident && (dir & 1)) {
                            // Park the value in this row's (already consumed) x/q staging
                            // slots: 32 + 32 bytes hold the 16 fp32 outputs of the token.
                            mdef |= 1u << (2 * mt + h);
                            *reinterpret_cast<float2*>(Xs + row * 32 + 8 * qt4) = o_lo;
                            *reinterpret_cast<float2*>(Qs + row * 32 + 8 * qt4) = o_hi;
                        } else if (KIND == kKindRows && (coincident || partner_later)) {
                            *reinterpret_cast<float2*>(op) = o_lo;
                            *reinterpret_cast<float2*>(op + 8) = o_hi;
                        } else {
                            const float2 p_lo = *reinterpret_cast<const float2*>(op);
                            const float2 p_hi = *reinterpret_cast<const float2*>(op + 8);
                            *reinterpret_cast<float2*>(op) = make_float2(p_lo.x + o_lo.x, p_lo.y + o_lo.y);
                            *reinterpret_cast<float2*>(op + 8) = make_float2(p_hi.x + o_hi.x, p_hi.y + o_hi.y);
                        }
                    } else {
                        if (t < p.L) {
                            XT* yo = mt_y[mt] + t * D + 2 * qt4;
                            *reinterpret_cast<__nv_bfloat162*>(yo) = __floats2bfloat162_rn(yv[0], yv[1]);
                            *reinterpret_cast<__nv_bfloat162*>(yo + 8) = __floats2bfloat162_rn(yv[2], yv[3]);
                        }
                    }
                }
            }
            __syncwarp();  // raw k~ / v rows of this warp's tokens are staged
            if (p1_on && p1_tok < count) {
                const float* Sc = S + (size_t)p1_slot * SROWS * SP;
                float* krow = Kt + (size_t)tid * SP;
                float* drow = Dt + (size_t)tid * SP;
                float xv[D], kr[D], vv[D];
                xc.to_float(xv);
                float kn = 0.f;
#pragma unroll
                for (int i = 0; i < D; i += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(krow + i);
                    const float4 v4 = *reinterpret_cast<const float4*>(drow + i);
                    kr[i] = k4.x; kr[i + 1] = k4.y; kr[i + 2] = k4.z; kr[i + 3] = k4.w;
                    vv[i] = v4.x; vv[i + 1] = v4.y; vv[i + 2] = v4.z; vv[i + 3] = v4.w;
                }
#pragma unroll
                for (int i = 0; i < D; ++i) kn = fmaf(kr[i], kr[i], kn);
                const float kinv = key_inv_norm(kn);
                float ke = 0.f, dn2 = 0.f, ep = 0.f, ap = 0.f;
                const float* ev = Sc + 3 * D * SP;
                const float* avp = Sc + (3 * D + 1) * SP;
#pragma unroll
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
#pragma unroll
                for (int i = 0; i < D; i += 4) {
                    *reinterpret_cast<float4*>(krow + i) = make_float4(kr[i], kr[i + 1], kr[i + 2], kr[i + 3]);
                    *reinterpret_cast<float4*>(drow + i) = make_float4(vv[i], vv[i + 1], vv[i + 2], vv[i + 3]);
                }
                const float2 gg = token_gate_scalars(p.k, ep, ap, ke, dn2);
                const float eff = gg.x, alpha = gg.y;
                EFF[tid] = eff;
                ALP[tid] = alpha;
            }
        } else if (p1_on && p1_tok < count) {
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
            const float kinv = key_inv_norm(kn);
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
            const float2 gg = token_gate_scalars(p.k, ep, ap, ke, dn2);
            const float eff = gg.x, alpha = gg.y;
            EFF[row] = eff;
            ALP[row] = alpha;
        }
        __syncthreads();
        if constexpr (MMA && kSpatial) {
            if (mdef) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        if (mdef & (1u << (2 * mt + h))) {
                            const int row = wrp * 32 + mt * 16 + qg + 8 * h;
                            const int tin = (j << lt) + (row & (tile - 1));
                            float* op = mt_out[mt] + (int64_t)scan_pixel(mt_ch[mt].dir, c, tin, p.H, p.W) * p.C + 2 * qt4;
                            const float2 o_lo = *reinterpret_cast<const float2*>(Xs + row * 32 + 8 * qt4);
                            const float2 o_hi = *reinterpret_cast<const float2*>(Qs + row * 32 + 8 * qt4);
                            const float2 p_lo = *reinterpret_cast<const float2*>(op);
                            const float2 p_hi = *reinterpret_cast<const float2*>(op + 8);
                            *reinterpret_cast<float2*>(op) = make_float2(p_lo.x + o_lo.x, p_lo.y + o_lo.y);
                            *reinterpret_cast<float2*>(op + 8) = make_float2(p_hi.x + o_hi.x, p_hi.y + o_hi.y);
                        }
            }
        }
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
                    if constexpr (MMA) {
                        const int r = task - slot * SROWS;
                        if (r < 3 * D) write_splits16(Mb + (size_t)slot * kSplits * 48 * 32, r, acc);
                    }
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
