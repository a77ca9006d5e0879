// Warp-per-chain SRNL scan for head_dim 16 with bf16 inputs (the inference hot path).
//
// One warp owns one chain (a (batch, direction, head) scan) for its whole length.  A CTA holds
// four warps and never synchronizes them before its end, so each warp advances on its own and
// the SM hides one warp's latency behind the others:
//   kKindBoth  the four scans of one (batch, head), each writing its own fp32 plane (scan 0
//              `out`, scans 1-3 the three planes of `aux`); the CTA then sums the four planes
//              of its (batch, head) into `out`, or writes (final dtype)(sum + addend) to `fin`.
//   kKindSeq   four independent packed-sequence chains.
//
// Per chunk (chunk-start state S = [M_m; M_v; M_k; e^T; a^T], gain G reset to I):
//   P1  tokens in steps of 32 (two 16-row MMA tiles):
//       - the step's x and raw q token rows arrive in shared memory by asynchronous copies
//         issued during the previous step, and feed the MMAs through ldmatrix;
//       - k~ = M_k x, v = M_v x and M_m q_raw run as bf16 m16n8k16 tensor-core MMAs against
//         the three-way bf16 split of the fp32 memories (fp32 accumulate, 24-bit operands);
//         y = (M_m q_raw) / ||q_raw|| (models/srnl_core/csrc/inference_recurrence.cuh:40-60);
//       - each token's own lane (a lane pair, in steps of at most 16 tokens) finishes the key
//         norm, the eta/alpha gates, the injection cap and the spectral clamp
//         (inference_recurrence.cuh:60-90, memory.cuh:219-233), and k_t . k_{t+1} for the
//         lookahead below.
//   P2  the gain recurrence r_t = (k_t - v_t) + G k_t, G <- alpha_t G - eta_t r_t k_t^T
//       (inference_recurrence.cuh:92-106), two lanes per row of G, eight columns each.
//       r_{t+1} is formed as d_{t+1} + alpha_t (G k_{t+1}) - u_t (k_t . k_{t+1}) with
//       u_t = eta_t r_t, so the dot product for token t+1 runs beside the update of token t
//       and the serial dependence per token is one FMA and one multiply.
//   P3  S <- S G (inference_recurrence.cuh:110-135) as tensor-core MMAs over split operands
//       (6 of the 9 split products; the dropped ones are below 2^-24 relative).
// The memories, e and a live only as their three exact bf16 parts (the truncation split: the
// parts sum to the fp32 value exactly); x.e and x.a come out of the projection MMA as an extra
// column tile.
//
// Spatial output: every scan stores w_d (y + s_d x) for each pixel it visits into its own
// plane (one plain store per pixel and scan, no read-back, no ordering between scans); the
// four planes are summed in a fixed order at the CTA's end, so results are deterministic.
#pragma once

#include "f32x2.cuh"
#include "srnl_scan.cuh"

namespace vh {
namespace wpc {

#ifndef VH_WPC_MIN_BLOCKS
#define VH_WPC_MIN_BLOCKS 4
#endif
#ifndef VH_WPC_MIN_BLOCKS_16
#define VH_WPC_MIN_BLOCKS_16 5
#endif

constexpr int kD = 16;
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kTile = 32;  // tokens per step (two 16-row MMA tiles)
constexpr int kKP = 20;    // padded row stride (floats) of the per-token key rows: 80-byte rows
                           // keep the one-token-per-lane float4 accesses free of bank conflicts

// Per-warp (per-chain) shared memory for steps of TILE tokens (32, or 16 when every chunk
// has at most 16 tokens: less shared memory per chain, so five CTAs fit an SM).
template <int TILE>
struct alignas(16) ChainSmemT {
    static constexpr int kTileT = TILE;
    // The stacked state as three exact bf16 parts: rows 0-15 M_m, 16-31 M_v, 32-47 M_k,
    // 48 e (learning-rate memory), 49 a (retention memory), 50-63 zero.
    unsigned char mb[kSplits][64][32];
    float kt[TILE][kKP];                // raw k~, then the normalized key k
    float dt[TILE][kKP];                // raw v, then d = k - v
    float4 gate[TILE];                  // (x.e, x.a) then (eta_eff, alpha, k_t . k_{t+1}, -)
    float fw[2][kD];                    // spatial: this scan's fusion weight and skip per channel
    unsigned char xq[2][TILE][32];      // the step's x and raw q token rows (bf16, swizzled)
    static_assert(kSplits * 16 * 32 <= 2 * (int)sizeof(float) * TILE * kKP,
                  "gain parts must fit the key and value rows");
};
using ChainSmem = ChainSmemT<kTile>;

// The three bf16 parts of G (row-major, k x n) live in the key (and value) rows during the
// boundary refresh, when no token data is held there.
template <class CS>
__device__ __forceinline__ unsigned char* gain_parts(CS& cs, int k) {
    return reinterpret_cast<unsigned char*>(&cs.kt[0][0]) + k * 16 * 32;
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const unsigned char* p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const unsigned char* p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Exact three-way bf16 split of a pair of fp32 values by truncation: part k packs (lo, hi) of
// the top 8 significant bits left after parts 0..k-1, so x = part0 + part1 + part2 exactly.
// A part is the upper half of an fp32 word, so one byte permute packs a pair, and one packed
// subtraction (exact: it only clears the leading bits) removes it from both values.
__device__ __forceinline__ void split3(float lo, float hi, uint32_t (&parts)[kSplits]) {
    float2 v = make_float2(lo, hi);
#pragma unroll
    for (int k = 0; k < kSplits; ++k) {
        const uint32_t ul = __float_as_uint(v.x), uh = __float_as_uint(v.y);
        parts[k] = __byte_perm(ul, uh, 0x7632);
        if (k + 1 < kSplits)
            v = fsub2(v, make_float2(__uint_as_float(ul & 0xffff0000u), __uint_as_float(uh & 0xffff0000u)));
    }
}

// Stores one 16-value row of the stacked state as its three bf16 parts.
template <class CS>
__device__ __forceinline__ void put_row_splits(CS& cs, int r, const float* v) {
    uint32_t w[kSplits][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t parts[kSplits];
        split3(v[2 * i], v[2 * i + 1], parts);
#pragma unroll
        for (int k = 0; k < kSplits; ++k) w[k][i] = parts[k];
    }
#pragma unroll
    for (int k = 0; k < kSplits; ++k) {
        *reinterpret_cast<uint4*>(&cs.mb[k][0][0] + swz(r, 0)) = make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]);
        *reinterpret_cast<uint4*>(&cs.mb[k][0][0] + swz(r, 1)) = make_uint4(w[k][4], w[k][5], w[k][6], w[k][7]);
    }
}

struct Role {
    int b, dir, head, valid;
    float* plane;  // spatial: this scan's output plane
};

template <int KIND>
__device__ __forceinline__ Role warp_role(const ScanParams& p, int warp) {
    Role r;
    int idx;
    if (KIND == kKindSeq) {
        idx = blockIdx.x * kWarps + warp;
        r.dir = blockIdx.y;
    } else {
        idx = blockIdx.x;
        r.dir = warp;
    }
    r.valid = idx < p.B * p.heads;
    r.b = r.valid ? idx / p.heads : 0;
    r.head = r.valid ? idx % p.heads : 0;
    r.plane = warp == 0 || KIND == kKindSeq ? p.out : p.aux + (int64_t)(warp - 1) * p.B * p.ob;
    return r;
}

// The gain recurrence over the `count` tokens of one step (N > 0: exactly N, unrolled).
// Lane (row, half) holds G[row][8 half .. 8 half + 7] in g as four column pairs; the dot
// products and the update run as packed two-lane FMAs (lane pair (2i, 2i+1) of g[i]).
template <class CS>
__device__ __forceinline__ void load_key_half(const CS& cs, int t, int half, float2 (&k)[4]) {
    const float4 lo = *reinterpret_cast<const float4*>(&cs.kt[t][8 * half]);
    const float4 hi = *reinterpret_cast<const float4*>(&cs.kt[t][8 * half + 4]);
    k[0] = make_float2(lo.x, lo.y);
    k[1] = make_float2(lo.z, lo.w);
    k[2] = make_float2(hi.x, hi.y);
    k[3] = make_float2(hi.z, hi.w);
}

// G[row] . k over the whole row: this lane's eight columns, then the partner half's.
__device__ __forceinline__ float row_dot(const float2 (&g)[4], const float2 (&k)[4]) {
    float2 a = fmul2(g[0], k[0]);
    a = ffma2(g[1], k[1], a);
    a = ffma2(g[2], k[2], a);
    a = ffma2(g[3], k[3], a);
    float part = a.x + a.y;
    part += __shfl_xor_sync(0xffffffffu, part, 16);
    return part;
}

template <int N, class CS>
__device__ __forceinline__ void gain_pass(const CS& cs, int count, int row, int half, float2 (&g)[4]) {
    if (N > 0) count = N;
    float2 kc[4];
    load_key_half(cs, 0, half, kc);
    float4 gt = cs.gate[0];
    float u = gt.x * (row_dot(g, kc) + cs.dt[0][row]);
#pragma unroll (N > 0 ? N : 1)
    for (int t = 0; t < count; ++t) {
        const float alpha = gt.y, kk = gt.z;
        float2 kn[4];
        float unext = 0.f;
        if (t + 1 < count) {
            load_key_half(cs, t + 1, half, kn);
            gt = cs.gate[t + 1];
            // r_{t+1} = d_{t+1} + alpha_t (G_{t-1} k_{t+1}) - u_t (k_t . k_{t+1})
            const float r = fmaf(-u, kk, fmaf(alpha, row_dot(g, kn), cs.dt[t + 1][row]));
            unext = gt.x * r;
        }
        const float2 a2 = splat2(alpha), nu2 = splat2(-u);
#pragma unroll
        for (int i = 0; i < 4; ++i) g[i] = ffma2(nu2, kc[i], fmul2(a2, g[i]));
        if (t + 1 < count) {
#pragma unroll
            for (int i = 0; i < 4; ++i) kc[i] = kn[i];
        }
        u = unext;
    }
}

// Dispatches the gain recurrence to a fully unrolled body for the step lengths the
// VisionHOPE stages produce (chunks of 56, 28, 14 and 7 tokens in steps of at most 32).
template <class CS>
__device__ __forceinline__ void gain_step(const CS& cs, int count, int row, int half, float2 (&g)[4]) {
    if constexpr (CS::kTileT == 32) {
        switch (count) {
            case 32: gain_pass<32>(cs, count, row, half, g); return;
            case 28: gain_pass<28>(cs, count, row, half, g); return;
            case 24: gain_pass<24>(cs, count, row, half, g); return;
            default: break;
        }
    }
    switch (count) {
        case 14: gain_pass<14>(cs, count, row, half, g); break;
        case 7: gain_pass<7>(cs, count, row, half, g); break;
        default: gain_pass<0>(cs, count, row, half, g);
    }
}

// Gates of a step of at most 16 tokens, two lanes per token: lane (t, hf) holds channels
// 8 hf .. 8 hf + 7 of token t, and the pair combines its partial sums with one shuffle.
// k_t . k_{t+1} for the lookahead of the gain recurrence comes from the raw keys in the same
// pass: (k~_t . k~_{t+1}) / (||k~_t|| ||k~_{t+1}||).
template <class CS>
__device__ __forceinline__ void gates_two_lane(CS& cs, const ScanParams& p, int count, int lane) {
    const int t = lane & 15, hf = lane >> 4;
    const bool live = t < count, nxt = t + 1 < count;
    const int tt = live ? t : 0, tn = nxt ? t + 1 : 0;
    float2 k[4], v[4], kn[4];
    {
        const float4 a0 = *reinterpret_cast<const float4*>(&cs.kt[tt][8 * hf]);
        const float4 a1 = *reinterpret_cast<const float4*>(&cs.kt[tt][8 * hf + 4]);
        const float4 b0 = *reinterpret_cast<const float4*>(&cs.dt[tt][8 * hf]);
        const float4 b1 = *reinterpret_cast<const float4*>(&cs.dt[tt][8 * hf + 4]);
        const float4 c0 = *reinterpret_cast<const float4*>(&cs.kt[tn][8 * hf]);
        const float4 c1 = *reinterpret_cast<const float4*>(&cs.kt[tn][8 * hf + 4]);
        k[0] = make_float2(a0.x, a0.y); k[1] = make_float2(a0.z, a0.w);
        k[2] = make_float2(a1.x, a1.y); k[3] = make_float2(a1.z, a1.w);
        v[0] = make_float2(b0.x, b0.y); v[1] = make_float2(b0.z, b0.w);
        v[2] = make_float2(b1.x, b1.y); v[3] = make_float2(b1.z, b1.w);
        kn[0] = make_float2(c0.x, c0.y); kn[1] = make_float2(c0.z, c0.w);
        kn[2] = make_float2(c1.x, c1.y); kn[3] = make_float2(c1.z, c1.w);
    }
    const float2 raw = *reinterpret_cast<const float2*>(&cs.gate[tt]);
    __syncwarp();  // every raw row is read before any lane overwrites its own
    float2 skk = fmul2(k[0], k[0]), snn = fmul2(kn[0], kn[0]), skn = fmul2(k[0], kn[0]);
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        skk = ffma2(k[i], k[i], skk);
        snn = ffma2(kn[i], kn[i], snn);
        skn = ffma2(k[i], kn[i], skn);
    }
    float ss = skk.x + skk.y, sn = snn.x + snn.y, sx = skn.x + skn.y;
    ss += __shfl_xor_sync(0xffffffffu, ss, 16);
    sn += __shfl_xor_sync(0xffffffffu, sn, 16);
    sx += __shfl_xor_sync(0xffffffffu, sx, 16);
    const float kinv = key_inv_norm(ss), kinvn = key_inv_norm(sn);
    const float2 kinv2 = splat2(kinv);
    float2 ke2 = splat2(0.f), dn2 = splat2(0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        k[i] = fmul2(k[i], kinv2);
        v[i] = fadd2(k[i], make_float2(-v[i].x, -v[i].y));  // d = k - v
        ke2 = ffma2(k[i], k[i], ke2);
        dn2 = ffma2(v[i], v[i], dn2);
    }
    float ke = ke2.x + ke2.y, dns = dn2.x + dn2.y;
    ke += __shfl_xor_sync(0xffffffffu, ke, 16);
    dns += __shfl_xor_sync(0xffffffffu, dns, 16);
    if (live) {
        *reinterpret_cast<float4*>(&cs.kt[t][8 * hf]) = make_float4(k[0].x, k[0].y, k[1].x, k[1].y);
        *reinterpret_cast<float4*>(&cs.kt[t][8 * hf + 4]) = make_float4(k[2].x, k[2].y, k[3].x, k[3].y);
        *reinterpret_cast<float4*>(&cs.dt[t][8 * hf]) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
        *reinterpret_cast<float4*>(&cs.dt[t][8 * hf + 4]) = make_float4(v[2].x, v[2].y, v[3].x, v[3].y);
        const float2 g = token_gate_scalars(p.k, raw.x, raw.y, ke, dns);
        if (hf == 0) cs.gate[t] = make_float4(g.x, g.y, nxt ? sx * kinv * kinvn : 0.f, 0.f);
    }
}

template <bool kSpatial, int TILE>
__device__ __forceinline__ void scan_chain(const ScanParams& p, ChainSmemT<TILE>& cs, const Role& ro) {
    using bf16 = __nv_bfloat16;
    const int lane = threadIdx.x & 31;
    const int qg = lane >> 2, qt = lane & 3;  // MMA fragment coordinates
    const int dir = ro.dir;

    // ---- state set-up: split memories, e/a, and this lane's fusion weights -------------
    const int64_t sidx = p.mem_per_chain ? ((int64_t)ro.b * p.R + dir) * p.heads + ro.head
                                         : (int64_t)dir * p.heads + ro.head;
    for (int r = lane; r < 64; r += 32) {
        float v[kD];
        if (r < 48) {
            const float* src = r < 16 ? p.Mm + (sidx * kD + r) * kD
                             : r < 32 ? p.Mv + (sidx * kD + r - 16) * kD
                                      : p.Mk + (sidx * kD + r - 32) * kD;
#pragma unroll
            for (int i = 0; i < kD; i += 4) {
                const float4 f = *reinterpret_cast<const float4*>(src + i);
                v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
            }
        } else {
            const float* src = r == 48 ? p.Me + sidx * kD : p.Ma + sidx * kD;
#pragma unroll
            for (int i = 0; i < kD; ++i) v[i] = r < 50 ? src[i] : 0.f;
        }
        put_row_splits(cs, r, v);
    }
    if constexpr (kSpatial) {
        if (lane < kD) {
            const int c = ro.head * kD + lane;
            cs.fw[0][lane] = p.weight[dir * p.C + c];
            cs.fw[1][lane] = p.skip[(p.skip_per_dir ? dir * p.C : 0) + c];
        }
    }
    __syncwarp();

    int Lc, nchunks;
    if (kSpatial) {
        Lc = dir < 2 ? p.W : p.H;
        nchunks = dir < 2 ? p.H : p.W;
    } else {
        Lc = p.chunk[dir];
        nchunks = (p.L + Lc - 1) / Lc;
    }
    const int tpc = (Lc + TILE - 1) / TILE;  // steps per chunk
    const int last_count = Lc - (tpc - 1) * TILE;
    const int mtiles_last = (last_count + 15) >> 4;

    // ---- input addressing ------------------------------------------------------------
    const bf16* xbase;
    const bf16* qbase;
    int64_t xts, qts;
    float* obase = nullptr;
    bf16* ybase = nullptr;
    if constexpr (kSpatial) {
        xbase = static_cast<const bf16*>(p.x) + ro.b * p.xb + ro.head * p.xh + (p.remap ? 0 : dir * p.xd);
        qbase = static_cast<const bf16*>(p.q) + ro.b * p.qb + ro.head * p.qh + (p.remap ? 0 : dir * p.qd);
        xts = p.xt;
        qts = p.qt;
        obase = ro.plane + ro.b * p.ob + ro.head * kD + 2 * qt;
    } else {
        const int64_t chain = ((int64_t)ro.b * p.R + dir) * p.heads + ro.head;
        xbase = static_cast<const bf16*>(p.x) + chain * p.L * kD;
        qbase = static_cast<const bf16*>(p.q) + ((int64_t)ro.b * p.R + dir) * p.L * p.C + ro.head * kD;
        xts = kD;
        qts = p.C;
        ybase = static_cast<bf16*>(p.y) + chain * p.L * kD + 2 * qt;
    }
    // Pixel visited at token `tin` of chunk `c` is pb + c * pc_step + tin * pt_step (the four
    // scan orders of models/operator.py:79-86 as linear maps); the source element read is the
    // pixel when the input is one image (remap) and the scan position c * Lc + tin otherwise.
    int pb = 0, pc_step = 0, pt_step = 0;
    if constexpr (kSpatial) {
        const int last = p.H * p.W - 1;
        switch (dir) {
            case 0: pb = 0; pc_step = p.W; pt_step = 1; break;
            case 1: pb = last; pc_step = -p.W; pt_step = -1; break;
            case 2: pb = 0; pc_step = 1; pt_step = p.W; break;
            default: pb = last; pc_step = -1; pt_step = -p.W; break;
        }
    }
    const bool img_src = kSpatial && p.remap;
    const int sb = img_src ? pb : 0, sc_step = img_src ? pc_step : Lc, st_step = img_src ? pt_step : 1;

    // The x and raw q rows of a step go to shared memory as 16-byte asynchronous copies (two
    // per token row, zeros past the chunk or sequence end, as the reference pads:
    // models/srnl_core/chunk.py:202-206); the MMA fragments are then read with ldmatrix.
    auto prefetch = [&](int c, int j) {
        const int cb = sb + c * sc_step;
#pragma unroll
        for (int u = 0; u < TILE / 8; ++u) {
            const int id = u * 32 + lane;  // 4 TILE chunks: tensor, token, half
            const int tensor = id / (2 * TILE), tok = (id >> 1) & (TILE - 1), half = id & 1;
            const int tin = j * TILE + tok;
            const bool ok = tin < Lc && (kSpatial || (int64_t)c * Lc + tin < p.L);
            const int64_t s = cb + tin * st_step;
            const bf16* src = tensor ? qbase + s * qts : xbase + s * xts;
            cp_async16_zfill(&cs.xq[tensor][0][0] + swz(tok, half), ok ? src + 8 * half : xbase, ok);
        }
        cp_async_commit();
    };
    prefetch(0, 0);

    const int p2_row = lane & 15, p2_half = lane >> 4;
    float2 g8[4];  // this lane's half row of G as column pairs

    for (int c = 0; c < nchunks; ++c) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            g8[i] = make_float2(p2_half * 8 + 2 * i == p2_row ? 1.f : 0.f, p2_half * 8 + 2 * i + 1 == p2_row ? 1.f : 0.f);
        for (int j = 0; j < tpc; ++j) {
            const int count = j + 1 < tpc ? TILE : last_count;
            const int mtiles = j + 1 < tpc ? TILE / 16 : mtiles_last;
            cp_async_wait<0>();
            __syncwarp();

            // ---------------------------- P1: projections -------------------------------
#pragma unroll
            for (int mt = 0; mt < TILE / 16; ++mt) {
                if (mt >= mtiles) break;  // warp-uniform
                float ck[2][4] = {}, cv[2][4] = {}, cy[2][4] = {}, cea[4] = {};
                // A fragments: {row qg, row qg+8} x {channels 2qt.., 8+2qt..}
                uint32_t A_x[4], A_q[4];
                ldsm_x4(A_x, &cs.xq[0][0][0] + swz(mt * 16 + (lane & 15), lane >> 4));
                ldsm_x4(A_q, &cs.xq[1][0][0] + swz(mt * 16 + (lane & 15), lane >> 4));
                const int brow = (lane & 7) + ((lane >> 4) << 3), bhalf = (lane >> 3) & 1;
#pragma unroll
                for (int k = 0; k < kSplits; ++k) {
                    uint32_t bm[4], bv[4], bk[4];
                    ldsm_x4(bm, &cs.mb[k][0][0] + swz(brow, bhalf));
                    ldsm_x4(bv, &cs.mb[k][0][0] + swz(16 + brow, bhalf));
                    ldsm_x4(bk, &cs.mb[k][0][0] + swz(32 + brow, bhalf));
                    mma_16816(cy[0], A_q, bm[0], bm[1]);
                    mma_16816(cy[1], A_q, bm[2], bm[3]);
                    mma_16816(cv[0], A_x, bv[0], bv[1]);
                    mma_16816(cv[1], A_x, bv[2], bv[3]);
                    mma_16816(ck[0], A_x, bk[0], bk[1]);
                    mma_16816(ck[1], A_x, bk[2], bk[3]);
                    uint32_t bea[2];  // rows 48-55: e, a and zeros -> columns (x.e, x.a)
                    ldsm_x2(bea, &cs.mb[k][0][0] + swz(48 + (lane & 7), (lane >> 3) & 1));
                    mma_16816(cea, A_x, bea[0], bea[1]);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // Lane (qg, qt) holds channels {2qt, 2qt+1, 8+2qt, 9+2qt} of token row qg + 8h.
                    const int row = mt * 16 + qg + 8 * h;
                    const float2 x01 = bf2_to_f2(A_x[h]), x23 = bf2_to_f2(A_x[2 + h]);
                    const float2 q01 = bf2_to_f2(A_q[h]), q23 = bf2_to_f2(A_q[2 + h]);
                    *reinterpret_cast<float2*>(&cs.kt[row][2 * qt]) = make_float2(ck[0][2 * h], ck[0][2 * h + 1]);
                    *reinterpret_cast<float2*>(&cs.kt[row][8 + 2 * qt]) = make_float2(ck[1][2 * h], ck[1][2 * h + 1]);
                    *reinterpret_cast<float2*>(&cs.dt[row][2 * qt]) = make_float2(cv[0][2 * h], cv[0][2 * h + 1]);
                    *reinterpret_cast<float2*>(&cs.dt[row][8 + 2 * qt]) = make_float2(cv[1][2 * h], cv[1][2 * h + 1]);
                    const float qs = quad_sum(q01.x * q01.x + q01.y * q01.y + q23.x * q23.x + q23.y * q23.y);
                    if (qt == 0) *reinterpret_cast<float2*>(&cs.gate[row]) = make_float2(cea[2 * h], cea[2 * h + 1]);
                    // 1 / max(||q||, 1e-12) (inference_recurrence.cuh:45)
                    const float qinv = rsqrtf(fmaxf(qs, 1e-24f));
                    const float y0 = cy[0][2 * h] * qinv, y1 = cy[0][2 * h + 1] * qinv;
                    const float y2 = cy[1][2 * h] * qinv, y3 = cy[1][2 * h + 1] * qinv;
                    if constexpr (kSpatial) {
                        const float2 wl = *reinterpret_cast<const float2*>(&cs.fw[0][2 * qt]);
                        const float2 wh = *reinterpret_cast<const float2*>(&cs.fw[0][8 + 2 * qt]);
                        const float2 sl = *reinterpret_cast<const float2*>(&cs.fw[1][2 * qt]);
                        const float2 sh = *reinterpret_cast<const float2*>(&cs.fw[1][8 + 2 * qt]);
                        if (row < count) {  // this scan's plane: w_d (y + s_d x) for the pixel
                            float* op = obase + (int64_t)(pb + c * pc_step + (j * TILE + row) * pt_step) * p.C;
                            *reinterpret_cast<float2*>(op) =
                                make_float2(wl.x * (y0 + sl.x * x01.x), wl.y * (y1 + sl.y * x01.y));
                            *reinterpret_cast<float2*>(op + 8) =
                                make_float2(wh.x * (y2 + sh.x * x23.x), wh.y * (y3 + sh.y * x23.y));
                        }
                    } else {
                        const int64_t t = (int64_t)c * Lc + j * TILE + row;
                        if (row < count && t < p.L) {
                            bf16* yo = ybase + t * kD;
                            *reinterpret_cast<uint32_t*>(yo) = pack_bf2(y0, y1);
                            *reinterpret_cast<uint32_t*>(yo + 8) = pack_bf2(y2, y3);
                        }
                    }
                }
            }
            __syncwarp();  // every lane's fragments of this step are read: refill the tile
            if (j + 1 < tpc) prefetch(c, j + 1);
            else if (c + 1 < nchunks) prefetch(c + 1, 0);

            // ------------------ P1: per-token gates ------------------------------------------
            if constexpr (TILE == 16) {  // two lanes per token
                gates_two_lane(cs, p, count, lane);
                __syncwarp();
            } else {  // one lane per token
                float2 kr[kD / 2];
                if (lane < count) {
                    float2 vv[kD / 2];
#pragma unroll
                    for (int i = 0; i < kD; i += 4) {
                        const float4 k4 = *reinterpret_cast<const float4*>(&cs.kt[lane][i]);
                        const float4 v4 = *reinterpret_cast<const float4*>(&cs.dt[lane][i]);
                        kr[i / 2] = make_float2(k4.x, k4.y);
                        kr[i / 2 + 1] = make_float2(k4.z, k4.w);
                        vv[i / 2] = make_float2(v4.x, v4.y);
                        vv[i / 2 + 1] = make_float2(v4.z, v4.w);
                    }
                    float2 kn2 = fmul2(kr[0], kr[0]);
#pragma unroll
                    for (int i = 1; i < kD / 2; ++i) kn2 = ffma2(kr[i], kr[i], kn2);
                    const float kinv = key_inv_norm(kn2.x + kn2.y);
                    const float2 kinv2 = splat2(kinv);
                    float2 ke2 = splat2(0.f), dn2 = splat2(0.f);
#pragma unroll
                    for (int i = 0; i < kD / 2; ++i) {
                        kr[i] = fmul2(kr[i], kinv2);
                        vv[i] = fadd2(kr[i], make_float2(-vv[i].x, -vv[i].y));  // d = k - v
                        ke2 = ffma2(kr[i], kr[i], ke2);
                        dn2 = ffma2(vv[i], vv[i], dn2);
                    }
#pragma unroll
                    for (int i = 0; i < kD; i += 4) {
                        *reinterpret_cast<float4*>(&cs.kt[lane][i]) = make_float4(kr[i / 2].x, kr[i / 2].y, kr[i / 2 + 1].x, kr[i / 2 + 1].y);
                        *reinterpret_cast<float4*>(&cs.dt[lane][i]) = make_float4(vv[i / 2].x, vv[i / 2].y, vv[i / 2 + 1].x, vv[i / 2 + 1].y);
                    }
                    const float ke = ke2.x + ke2.y;
                    const float2 raw = *reinterpret_cast<const float2*>(&cs.gate[lane]);
                    const float2 gg = token_gate_scalars(p.k, raw.x, raw.y, ke, dn2.x + dn2.y);
                    const float eff = gg.x, alpha = gg.y;
                    *reinterpret_cast<float2*>(&cs.gate[lane]) = make_float2(eff, alpha);
                }
                __syncwarp();
                if (lane + 1 < count) {  // k_t . k_{t+1} for the lookahead of the gain recurrence
                    float2 kk2 = splat2(0.f);
#pragma unroll
                    for (int i = 0; i < kD; i += 4) {
                        const float4 k4 = *reinterpret_cast<const float4*>(&cs.kt[lane + 1][i]);
                        kk2 = ffma2(kr[i / 2], make_float2(k4.x, k4.y), kk2);
                        kk2 = ffma2(kr[i / 2 + 1], make_float2(k4.z, k4.w), kk2);
                    }
                    cs.gate[lane].z = kk2.x + kk2.y;
                }

                __syncwarp();
            }

            // ------------------ P2: gain recurrence ---------------------------------------------
            gain_step(cs, count, p2_row, p2_half, g8);
            __syncwarp();  // P1 of the next step overwrites kt/dt/gate
        }

        if (c + 1 == nchunks) break;
        // ------------------ P3: S <- S G on tensor cores ------------------------------------
        {
            uint32_t gp[kSplits][2][2];  // this lane's G row segment, split (8 values = 4 pairs)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t parts[kSplits];
                split3(g8[i].x, g8[i].y, parts);
#pragma unroll
                for (int k = 0; k < kSplits; ++k) gp[k][i >> 1][i & 1] = parts[k];
            }
#pragma unroll
            for (int k = 0; k < kSplits; ++k)
                *reinterpret_cast<uint4*>(gain_parts(cs, k) + swz(p2_row, p2_half)) =
                    make_uint4(gp[k][0][0], gp[k][0][1], gp[k][1][0], gp[k][1][1]);
            __syncwarp();
            uint32_t bg[kSplits][4];
#pragma unroll
            for (int k = 0; k < kSplits; ++k) ldsm_x4_trans(bg[k], gain_parts(cs, k) + swz(lane & 15, lane >> 4));
            // Products kept: (A part, G part) in {(0,0),(0,1),(1,0),(0,2),(2,0),(1,1)}.
            constexpr int kPa[6] = {0, 0, 1, 0, 2, 1};
            constexpr int kPg[6] = {0, 1, 0, 2, 0, 1};
            float acc[4][2][4] = {};
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {  // rows 0-47 memories, 48-63 e, a and zeros
                uint32_t am[kSplits][4];
#pragma unroll
                for (int k = 0; k < kSplits; ++k)
                    ldsm_x4(am[k], &cs.mb[k][0][0] + swz(mt * 16 + (lane & 15), lane >> 4));
#pragma unroll
                for (int q = 0; q < 6; ++q) {
                    mma_16816(acc[mt][0], am[kPa[q]], bg[kPg[q]][0], bg[kPg[q]][1]);
                    mma_16816(acc[mt][1], am[kPa[q]], bg[kPg[q]][2], bg[kPg[q]][3]);
                }
            }
            __syncwarp();  // every lane has read the old state parts
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (mt == 3 && h == 1) break;  // rows 56-63 are zero and stay zero
                    const int r = mt * 16 + qg + 8 * h;
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        uint32_t parts[kSplits];
                        split3(acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1], parts);
#pragma unroll
                        for (int k = 0; k < kSplits; ++k)
                            *reinterpret_cast<uint32_t*>(&cs.mb[k][0][0] + swz(r, nt) + 4 * qt) = parts[k];
                    }
                }
            __syncwarp();
        }
    }
}

// Stores four consecutive channels of the final output in its dtype.
__device__ __forceinline__ void store_final4(void* base, int dtype, int64_t off, float4 v) {
    if (dtype == VH_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(base) + off) = v;
    } else if (dtype == VH_BF16) {
        store4(static_cast<__nv_bfloat16*>(base) + off, v);
    } else {
        store4(static_cast<__half*>(base) + off, v);
    }
}

// End of a kKindBoth CTA: sum the four scans' planes of (b, head) in a fixed order into `out`,
// or write (final dtype)(sum + addend).  The loads of four pixel groups are issued before any
// store.
__device__ __forceinline__ void fold_planes(const ScanParams& p, int b, int head) {
    constexpr int kU = 4;
    const int n = p.H * p.W * 4;  // float4 groups of this head's 16 channels
    const int64_t ps = (int64_t)p.B * p.ob;  // elements between the aux planes
    float* A = p.out + b * p.ob + head * kD;
    const float* P1 = p.aux + b * p.ob + head * kD;
    const __nv_bfloat16* add =
        p.addend ? static_cast<const __nv_bfloat16*>(p.addend) + b * p.ab + head * kD : nullptr;
    for (int i0 = threadIdx.x; i0 < n; i0 += kThreads * kU) {
        float4 s[kU];
        int64_t off[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int i = i0 + u * kThreads;
            off[u] = (int64_t)(i >> 2) * p.C + (i & 3) * 4;
            s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n) {
                const float4 a = *reinterpret_cast<const float4*>(A + off[u]);
                const float4 c1 = *reinterpret_cast<const float4*>(P1 + off[u]);
                const float4 c2 = *reinterpret_cast<const float4*>(P1 + ps + off[u]);
                const float4 c3 = *reinterpret_cast<const float4*>(P1 + 2 * ps + off[u]);
                s[u] = make_float4(((a.x + c1.x) + c2.x) + c3.x, ((a.y + c1.y) + c2.y) + c3.y,
                                   ((a.z + c1.z) + c2.z) + c3.z, ((a.w + c1.w) + c2.w) + c3.w);
                if (add) {
                    const float4 e = load4(add + off[u]);
                    s[u] = make_float4(s[u].x + e.x, s[u].y + e.y, s[u].z + e.z, s[u].w + e.w);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (i0 + u * kThreads >= n) break;
            if (p.fin) store_final4(p.fin, p.fin_dtype, b * p.fb + head * kD + off[u], s[u]);
            else *reinterpret_cast<float4*>(A + off[u]) = s[u];
        }
    }
}

template <int KIND, int TILE>
__global__ void __launch_bounds__(kThreads, TILE == 16 ? VH_WPC_MIN_BLOCKS_16 : VH_WPC_MIN_BLOCKS)
    srnl_warp_kernel(const ScanParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    ChainSmemT<TILE>& cs = reinterpret_cast<ChainSmemT<TILE>*>(smem_raw)[warp];
    const Role ro = warp_role<KIND>(p, warp);
    if (ro.valid) scan_chain<KIND != kKindSeq, TILE>(p, cs, ro);
    if constexpr (KIND == kKindBoth) {
        __syncthreads();  // the four planes of this (b, head) are complete
        fold_planes(p, ro.b, ro.head);
    }
}

}  // namespace wpc
}  // namespace vh
