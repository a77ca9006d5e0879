// Chunk-parallel SRNL scan on the Blackwell tensor cores (head_dim 16, bf16 x and raw q).
//
// The warp-per-chain scan (srnl_warp.cuh) runs each chain's tokens through one warp, one
// token after the other, which leaves most of the GPU idle when a launch has few chains -- the
// dense 512 x 2048 configuration has 24 chains of 65 536 tokens at its first stage.  This kernel
// gives each chain a whole CTA of eight warps and runs a chunk's tokens in parallel:
//
//   load  the chunk's x and raw q rows arrive by TMA (cp.async.bulk.tensor, 32-byte swizzle)
//         from index-remapped tensor maps: rows of the channels-last image for scans 0/1,
//         columns (a box one pixel wide and up to 256 high) for scans 2/3, so no scan order is
//         ever materialised; the reversed scans load the same boxes and walk them backwards.
//         The next pass's tiles load while the current one computes (two buffers).
//   P1    projections on tcgen05: tokens on M (128 per MMA), the stacked chunk-start state
//         [M_m; M_v; M_k; e^T; a^T] on N (64 columns), K = 16 q channels then 16 x channels;
//         the fp32 state enters as three exact bf16 parts, so six MMAs per 128 tokens give
//         fp32-level projections, accumulated in TMEM.  Each thread then reads its token's
//         row of the accumulator (tcgen05.ld) and finishes, in registers: y = M_m q / ||q||
//         and its output, the key normalization, the eta/alpha gates, the soft injection cap
//         and the spectral clamp (models/srnl_core/csrc/inference_recurrence.cuh:40-90,
//         memory.cuh:219-233).
//   P2    the gain recurrence G_t = G_{t-1} (alpha_t I - eta_t k_t k_t^T) - eta_t d_t k_t^T
//         (d = k - v; inference_recurrence.cuh:92-106) is affine in G, so a segment of tokens
//         maps G_in to G_in P + Q.  Each warp runs one segment of the chunk and computes its
//         [P; Q] (32 rows of 16, one lane per row, from [I; 0]); the segments are then
//         composed in scan order, G <- G P_s + Q_s.
//   P3    the boundary refresh S <- S G (inference_recurrence.cuh:110-135) in fp32, and the
//         new state's bf16 parts written back as the next chunk's MMA operand.
// Chunks longer than 512 tokens run as several passes with G carried between them.
//
// Spatial output: each scan's CTA stores w_d (y + s_d x) for the pixels it visits into its own
// fp32 plane (scan 0 `out`, scans 1-3 the three `aux` planes); a second kernel sums the four
// planes in the fixed order ((p0 + p1) + p2) + p3 and writes out (or the final dtype with the
// addend), so results are deterministic.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "abi_util.h"
#include "f32x2.cuh"
#include "srnl_scan.cuh"
#include "tc_util.cuh"

namespace vh {
namespace tc {

constexpr int kD = 16;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kST = 128;        // tokens per MMA (M)
constexpr int kCols = 64;       // accumulator columns per MMA (N): 16 y, 16 v, 16 k~, x.e, x.a, zeros
constexpr int kBoxMax = 256;    // TMA box limit along the token dimension
constexpr int kRec = 20;        // floats per token record row (80-byte rows)
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s
constexpr uint32_t kIdesc = tcu::idesc_bf16_f32(kST, kCols);

// Tensor maps of one launch: [0] rows (scans 0/1) or token order, [1] columns (scans 2/3).
struct TcMaps {
    CUtensorMap x[2];
    CUtensorMap q[2];
};

// Launch-wide tile geometry (uniform over the chains of one launch).
struct TcGeom {
    int layout;       // 0 image (remap), 1 serialized scans [B, 4, L, C], 2 packed sequence
    int box_rows;     // tokens per TMA box along rows / token order
    int box_cols;     // tokens per TMA box along columns
};

// Shared-memory carve-up for passes of NST * 128 tokens (identical on host and device).
template <int NST>
struct TcSmem {
    static constexpr int kCap = NST * kST;
    static constexpr size_t kTile = size_t(kCap) * 32;  // one tensor's tile (bf16 rows of 16)
    static constexpr size_t TILES = 0;                   // [2 buffers][x, q][kCap][32 B]
    static constexpr size_t BOP = TILES + 4 * kTile;     // [q, x][3 parts][64 rows][32 B]
    static constexpr size_t S32 = BOP + 6 * 64 * 32;     // fp32 state [64][16]
    static constexpr size_t GB = S32 + 64 * 16 * 4;      // G [2][16][16]
    static constexpr size_t SEG = GB + 2 * 256 * 4;      // [8 warps][32 rows][16]
    static constexpr size_t RK = SEG + kWarps * 32 * 16 * 4;  // normalized keys [kCap][kRec]
    static constexpr size_t RD = RK + size_t(kCap) * kRec * 4;  // d = k - v [kCap][kRec]
    static constexpr size_t REA = RD + size_t(kCap) * kRec * 4;  // (eta_eff, alpha) [kCap]
    static constexpr size_t FW = REA + size_t(kCap) * 8;         // spatial weights, skips [2][16]
    static constexpr size_t BAR = FW + 2 * 16 * 4;               // mbarriers: tma[2], mma
    static constexpr size_t MISC = BAR + 3 * 8;                  // tmem base, abort flag
    static constexpr size_t kBytes = MISC + 16;
    static constexpr size_t kLaunch = kBytes + 1024;             // room to align the base to 1 KB
};

__device__ unsigned int g_tc_status;  // non-zero once a bounded wait gave up (cleared on read)

__device__ __forceinline__ int swz32(int row, int half) { return row * 32 + ((half ^ ((row >> 2) & 1)) << 4); }

__device__ __forceinline__ void tile_row(const unsigned char* tile, int row, float (&v)[16]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4 u = *reinterpret_cast<const uint4*>(tile + swz32(row, h));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = bf2_to_f2(w[i]);
            v[8 * h + 2 * i] = f.x;
            v[8 * h + 2 * i + 1] = f.y;
        }
    }
}

// Writes the three exact bf16 parts of one state value into the MMA operand rows (truncation
// split: part0 + part1 + part2 == v exactly).
__device__ __forceinline__ void put_parts(unsigned char* bop, int which, int row, int col, float v) {
#pragma unroll
    for (int k = 0; k < kSplits; ++k) {
        const uint32_t u = __float_as_uint(v);
        const unsigned short hi = static_cast<unsigned short>(u >> 16);
        unsigned char* part = bop + (size_t(which) * kSplits + k) * 64 * 32;
        *reinterpret_cast<unsigned short*>(part + swz32(row, col >> 3) + (col & 7) * 2) = hi;
        v -= __uint_as_float(u & 0xffff0000u);
    }
}

struct ChainInfo {
    int b, dir, head, chain, Lc, nchunks, reversed, mapi;
};

template <bool kSpatial>
__device__ __forceinline__ ChainInfo chain_info(const ScanParams& p) {
    ChainInfo ci;
    if (kSpatial) {
        ci.dir = blockIdx.x & 3;
        const int bh = blockIdx.x >> 2;
        ci.b = bh / p.heads;
        ci.head = bh - ci.b * p.heads;
        ci.chain = blockIdx.x;
        ci.Lc = ci.dir < 2 ? p.W : p.H;
        ci.nchunks = ci.dir < 2 ? p.H : p.W;
        ci.reversed = p.remap ? (ci.dir & 1) : 0;
        ci.mapi = p.remap ? (ci.dir >> 1) : 0;
    } else {
        ci.chain = blockIdx.x;  // (b, r, head)
        ci.head = ci.chain % p.heads;
        const int br = ci.chain / p.heads;
        ci.dir = br % p.R;
        ci.b = br / p.R;
        ci.Lc = p.chunk[ci.dir];
        ci.nchunks = (p.L + ci.Lc - 1) / ci.Lc;
        ci.reversed = 0;
        ci.mapi = 0;
    }
    return ci;
}

// Issues the TMA loads of one pass (x and q tiles) into `buf` and arms its barrier.
template <int NST, bool kSpatial>
__device__ __forceinline__ void issue_pass_loads(const ScanParams& p, const TcMaps& maps, const TcGeom& g,
                                                 const ChainInfo& ci, unsigned char* tiles, uint64_t* bar,
                                                 int buf, int c, int start, int n) {
    using S = TcSmem<NST>;
    const int bt = ci.mapi ? g.box_cols : g.box_rows;
    // Only tokens that exist are loaded: past a sequence's end the readback substitutes zero
    // tokens itself.  Every pass then needs one box, or boxes of 256 tokens (8 KB apart).
    int avail = n;
    if (!kSpatial) avail = max(0, min(n, p.L - (c * ci.Lc + start)));
    const int nbox = (avail + bt - 1) / bt;
    unsigned char* xt = tiles + size_t(buf) * 2 * S::kTile;
    unsigned char* qt = xt + S::kTile;
    tcu::mbar_arrive_expect_tx(bar, uint32_t(nbox) * bt * 32 * 2);
    const void* mx = &maps.x[ci.mapi];
    const void* mq = &maps.q[ci.mapi];
    for (int m = 0; m < nbox; ++m) {
        const int pos = start + m * bt;
        unsigned char* dx = xt + size_t(m) * bt * 32;
        unsigned char* dq = qt + size_t(m) * bt * 32;
        if (kSpatial && g.layout == 0) {
            if (ci.mapi == 0) {  // row h of image b: (channel, w, h, b)
                const int row = ci.dir == 0 ? c : p.H - 1 - c;
                tcu::tma_load_4d(dx, mx, bar, ci.head * kD, pos, row, ci.b);
                tcu::tma_load_4d(dq, mq, bar, ci.head * kD, pos, row, ci.b);
            } else {  // column w of image b: (channel, w, h, b) with a one-pixel-wide box
                const int col = ci.dir == 2 ? c : p.W - 1 - c;
                tcu::tma_load_4d(dx, mx, bar, ci.head * kD, col, pos, ci.b);
                tcu::tma_load_4d(dq, mq, bar, ci.head * kD, col, pos, ci.b);
            }
        } else if (kSpatial) {  // serialized scans [B, 4, L, C]: (channel, token, dir, b)
            const int tok = c * ci.Lc + pos;
            tcu::tma_load_4d(dx, mx, bar, ci.head * kD, tok, ci.dir, ci.b);
            tcu::tma_load_4d(dq, mq, bar, ci.head * kD, tok, ci.dir, ci.b);
        } else {  // packed x [chains, L, 16]; raw q [B*R, L, C]
            const int tok = c * ci.Lc + pos;
            tcu::tma_load_3d(dx, mx, bar, 0, tok, ci.chain);
            tcu::tma_load_3d(dq, mq, bar, ci.head * kD, tok, ci.b * p.R + ci.dir);
        }
    }
}

// Token gates of inference_recurrence.cuh:60-90 / memory.cuh:219-233 from the raw projections:
// k~ (kt) and v in, the normalized key in kt, d = k - v in v, (eta_eff, alpha) returned.
__device__ __forceinline__ float2 token_gates(const SrnlConsts& K, float (&kt)[16], float (&v)[16], float xe,
                                              float xa) {
    float kn2 = 0.f;
#pragma unroll
    for (int i = 0; i < kD; ++i) kn2 = fmaf(kt[i], kt[i], kn2);
    const float kinv = key_inv_norm(kn2);
    float ke = 0.f, dn2 = 0.f;
#pragma unroll
    for (int i = 0; i < kD; ++i) {
        kt[i] *= kinv;
        v[i] = kt[i] - v[i];
        ke = fmaf(kt[i], kt[i], ke);
        dn2 = fmaf(v[i], v[i], dn2);
    }
    return token_gate_scalars(K, xe, xa, ke, dn2);
}

template <int NST, bool kSpatial>
__global__ void __launch_bounds__(kThreads, NST == 4 ? 1 : 2)
    srnl_tc_kernel(const ScanParams p, const TcGeom g, const __grid_constant__ TcMaps maps) {
    using S = TcSmem<NST>;
    extern __shared__ unsigned char smem_dyn[];
    // The base rounded up to 1 KB (the swizzled operand tiles need it), as an offset from the
    // shared array itself: the compiler then keeps every derived pointer in the shared address
    // space (shared loads and stores, not generic ones).
    unsigned char* sm = smem_dyn + ((1024u - (tcu::smem_u32(smem_dyn) & 1023u)) & 1023u);
    unsigned char* tiles = sm + S::TILES;
    unsigned char* bop = sm + S::BOP;
    float* s32 = reinterpret_cast<float*>(sm + S::S32);
    float* gb = reinterpret_cast<float*>(sm + S::GB);
    float* seg = reinterpret_cast<float*>(sm + S::SEG);
    float* rk = reinterpret_cast<float*>(sm + S::RK);
    float* rd = reinterpret_cast<float*>(sm + S::RD);
    float2* rea = reinterpret_cast<float2*>(sm + S::REA);
    float* fw = reinterpret_cast<float*>(sm + S::FW);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BAR);  // [0], [1] tma buffers; [2] mma
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::MISC);
    int* abort_flag = reinterpret_cast<int*>(sm + S::MISC + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const ChainInfo ci = chain_info<kSpatial>(p);
    constexpr uint32_t kTmemCols = NST == 1 ? 64 : NST == 2 ? 128 : 256;

    // ---- set-up: state, operand parts, weights, barriers, TMEM ---------------------------------
    const int64_t sidx = p.mem_per_chain ? ((int64_t)ci.b * p.R + ci.dir) * p.heads + ci.head
                                         : (int64_t)ci.dir * p.heads + ci.head;
    for (int i = tid; i < 6 * 64 * 32 / 16; i += kThreads)
        reinterpret_cast<uint4*>(bop)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    for (int i = tid; i < 64 * kD; i += kThreads) {
        const int r = i >> 4, cc = i & 15;
        float v = 0.f;
        if (r < 16) v = p.Mm[(sidx * kD + r) * kD + cc];
        else if (r < 32) v = p.Mv[(sidx * kD + r - 16) * kD + cc];
        else if (r < 48) v = p.Mk[(sidx * kD + r - 32) * kD + cc];
        else if (r == 48) v = p.Me[sidx * kD + cc];
        else if (r == 49) v = p.Ma[sidx * kD + cc];
        s32[i] = v;
        if (r < 50) put_parts(bop, r < 16 ? 0 : 1, r, cc, v);
    }
    if (kSpatial && tid < kD) {
        const int ch = ci.head * kD + tid;
        fw[tid] = p.weight[ci.dir * p.C + ch];
        fw[16 + tid] = p.skip[(p.skip_per_dir ? ci.dir * p.C : 0) + ch];
    }
    if (tid == 0) {
        tcu::mbar_init(&bars[0], 1);
        tcu::mbar_init(&bars[1], 1);
        tcu::mbar_init(&bars[2], 1);
        *abort_flag = 0;
        tcu::fence_barrier_init();
    }
    if (warp == 0) tcu::tmem_alloc(tmem_slot, kTmemCols);
    tcu::fence_proxy_async_smem();  // operand parts written by threads, read by the MMA
    tcu::tc_fence_before_sync();
    __syncthreads();
    tcu::tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    const int cap = S::kCap;
    const int npass = (ci.Lc + cap - 1) / cap;
    auto pass_n = [&](int j) { return min(cap, ci.Lc - j * cap); };
    auto pass_start = [&](int j) { return ci.reversed ? ci.Lc - j * cap - pass_n(j) : j * cap; };
    const int total_passes = ci.nchunks * npass;
    // Loads in flight per buffer and the barrier parity that marks their completion (thread 0).
    bool tma_pending[2] = {false, false};
    uint32_t tma_parity[2] = {0u, 0u};
    if (tid == 0) {
        issue_pass_loads<NST, kSpatial>(p, maps, g, ci, tiles, &bars[0], 0, 0, pass_start(0), pass_n(0));
        tma_pending[0] = true;
        tma_parity[0] = 0u;
    }

    float* plane = nullptr;
    if (kSpatial) plane = (ci.dir == 0 ? p.out : p.aux + (int64_t)(ci.dir - 1) * p.B * p.ob) + ci.b * p.ob + ci.head * kD;

    int gp = 0;  // global pass index
    bool aborted = false;
    for (int c = 0; c < ci.nchunks && !aborted; ++c) {
        for (int j = 0; j < npass; ++j, ++gp) {
            const int n = pass_n(j), start = pass_start(j), buf = gp & 1;
            const unsigned char* xt = tiles + size_t(buf) * 2 * S::kTile;
            const unsigned char* qt = xt + S::kTile;
            // ---- TMA in, prefetch of the next pass, projections on the tensor cores ------------
            if (tid == 0) {
                bool ok = tcu::mbar_wait(&bars[buf], (gp >> 1) & 1, kWaitNs);
                if (ok) tma_pending[buf] = false;
                if (ok && gp + 1 < total_passes) {
                    const int jn = (j + 1 < npass) ? j + 1 : 0, cn = (j + 1 < npass) ? c : c + 1;
                    issue_pass_loads<NST, kSpatial>(p, maps, g, ci, tiles, &bars[buf ^ 1], buf ^ 1, cn, pass_start(jn),
                                                    pass_n(jn));
                    tma_pending[buf ^ 1] = true;
                    tma_parity[buf ^ 1] = ((gp + 1) >> 1) & 1;
                }
                if (ok) {
                    tcu::tc_fence_after_sync();
                    const int nst = (n + kST - 1) / kST;
                    for (int s = 0; s < nst; ++s) {
                        const uint32_t d = tmem + uint32_t(s * kCols);
                        const unsigned char* aq = qt + size_t(s) * kST * 32;
                        const unsigned char* ax = xt + size_t(s) * kST * 32;
#pragma unroll
                        for (int k = 0; k < kSplits; ++k)
                            tcu::mma_bf16(d, tcu::desc_kmajor_sw32(aq), tcu::desc_kmajor_sw32(bop + size_t(k) * 64 * 32),
                                          kIdesc, k > 0);
#pragma unroll
                        for (int k = 0; k < kSplits; ++k)
                            tcu::mma_bf16(d, tcu::desc_kmajor_sw32(ax),
                                          tcu::desc_kmajor_sw32(bop + size_t(kSplits + k) * 64 * 32), kIdesc, 1);
                    }
                    tcu::mma_commit(&bars[2]);
                    ok = tcu::mbar_wait(&bars[2], gp & 1, kWaitNs);
                }
                if (!ok) {
                    *abort_flag = 1;
                    atomicOr(&g_tc_status, 1u);
                }
            }
            if (__syncthreads_or(tid == 0 ? *abort_flag : 0)) {
                aborted = true;
                break;
            }
            tcu::tc_fence_after_sync();

            // ---- P1: one thread per token: gates and outputs from its accumulator row ----------
            const int qd = warp & 3;
            for (int s = warp >> 2; s * kST < n; s += 2) {
                const int i = s * kST + qd * 32 + lane;  // buffer row (image / token order)
                const uint32_t ta = tmem + (uint32_t(qd * 32) << 16) + uint32_t(s * kCols);
                float yv[16], vv[16], kv[16], ea[2];
                tcu::tmem_ld16(ta, yv);
                tcu::tmem_ld16(ta + 16, vv);
                tcu::tmem_ld16(ta + 32, kv);
                tcu::tmem_ld2(ta + 48, ea);
                tcu::tmem_wait_ld();
                if (i < n) {
                    const int t = ci.reversed ? n - 1 - i : i;  // pass-local scan index
                    const int64_t tok = (int64_t)c * ci.Lc + (int64_t)j * cap + t;
                    const bool real = kSpatial || tok < p.L;
                    if (!real) {  // padding past the sequence end: a zero token (chunk.py:202-206)
#pragma unroll
                        for (int e = 0; e < kD; ++e) { vv[e] = 0.f; kv[e] = 0.f; }
                        ea[0] = ea[1] = 0.f;
                    }
                    const float2 ga = token_gates(p.k, kv, vv, ea[0], ea[1]);
                    float* rkt = rk + t * kRec;
                    float* rdt = rd + t * kRec;
#pragma unroll
                    for (int e = 0; e < kD; e += 4) {
                        *reinterpret_cast<float4*>(rkt + e) = make_float4(kv[e], kv[e + 1], kv[e + 2], kv[e + 3]);
                        *reinterpret_cast<float4*>(rdt + e) = make_float4(vv[e], vv[e + 1], vv[e + 2], vv[e + 3]);
                    }
                    rea[t] = ga;
                    if (real) {
                        float qv[16];
                        tile_row(qt, i, qv);
                        float qs = 0.f;
#pragma unroll
                        for (int e = 0; e < kD; ++e) qs = fmaf(qv[e], qv[e], qs);
                        const float qinv = rsqrtf(fmaxf(qs, 1e-24f));  // 1 / max(||q||, 1e-12)
                        if (kSpatial) {
                            float xv[16];
                            tile_row(xt, i, xv);
                            int pix;
                            const int pos = start + i;  // position along this chunk's row / column
                            if (g.layout == 0) {
                                pix = ci.mapi == 0 ? (ci.dir == 0 ? c : p.H - 1 - c) * p.W + pos
                                                   : pos * p.W + (ci.dir == 2 ? c : p.W - 1 - c);
                            } else {
                                pix = scan_pixel(ci.dir, c, j * cap + t, p.H, p.W);
                            }
                            float* op = plane + (int64_t)pix * p.C;
#pragma unroll
                            for (int e = 0; e < kD; e += 4) {
                                float4 o;
                                o.x = fw[e] * (yv[e] * qinv + fw[16 + e] * xv[e]);
                                o.y = fw[e + 1] * (yv[e + 1] * qinv + fw[17 + e] * xv[e + 1]);
                                o.z = fw[e + 2] * (yv[e + 2] * qinv + fw[18 + e] * xv[e + 2]);
                                o.w = fw[e + 3] * (yv[e + 3] * qinv + fw[19 + e] * xv[e + 3]);
                                *reinterpret_cast<float4*>(op + e) = o;
                            }
                        } else {
                            __nv_bfloat16* yo = static_cast<__nv_bfloat16*>(p.y) + ((int64_t)ci.chain * p.L + tok) * kD;
                            uint32_t w[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const __nv_bfloat162 h = __floats2bfloat162_rn(yv[2 * e] * qinv, yv[2 * e + 1] * qinv);
                                w[e] = *reinterpret_cast<const uint32_t*>(&h);
                            }
                            reinterpret_cast<uint4*>(yo)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                            reinterpret_cast<uint4*>(yo)[1] = make_uint4(w[4], w[5], w[6], w[7]);
                        }
                    }
                }
            }
            tcu::tc_fence_before_sync();
            __syncthreads();  // records complete; TMEM and this buffer's tiles are free

            // ---- P2a: segment transitions [P; Q], one warp per segment, one lane per row --------
            // Passes of at most 128 tokens run at most four segments: the recurrence saturates
            // the FP32 pipe once eight warps share an SM (about 147 against 96 cycles per token
            // per warp with four), and each segment adds one step to the composition below.
            const int seg_len = n <= 128 ? max(16, (n + 3) / 4) : (n + kWarps - 1) / kWarps;
            const int nseg = (n + seg_len - 1) / seg_len;
            if (warp < nseg) {
                const int t0 = warp * seg_len, t1 = min(n, t0 + seg_len);
                float2 x8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    x8[e] = make_float2(lane == 2 * e ? 1.f : 0.f, lane == 2 * e + 1 ? 1.f : 0.f);
                const bool qrow = lane >= 16;
                // One token of the segment; blocks of 16 tokens run fully unrolled, so the next
                // tokens' key loads issue ahead of the current update (measured on B200, dense
                // stage 1: 2.84 against 3.27 ms with the plain loop).
                auto step = [&](int t) {
                    const float4* kr = reinterpret_cast<const float4*>(rk + t * kRec);
                    const float4 k0 = kr[0], k1 = kr[1], k2 = kr[2], k3 = kr[3];
                    const float2 k8[8] = {make_float2(k0.x, k0.y), make_float2(k0.z, k0.w), make_float2(k1.x, k1.y),
                                          make_float2(k1.z, k1.w), make_float2(k2.x, k2.y), make_float2(k2.z, k2.w),
                                          make_float2(k3.x, k3.y), make_float2(k3.z, k3.w)};
                    const float2 ga = rea[t];
                    const float dd = qrow ? rd[t * kRec + (lane - 16)] : 0.f;
                    float2 acc = fmul2(x8[0], k8[0]);
#pragma unroll
                    for (int e = 1; e < 8; ++e) acc = ffma2(x8[e], k8[e], acc);
                    const float u = -ga.x * ((acc.x + acc.y) + dd);
                    const float2 a2 = splat2(ga.y), u2 = splat2(u);
#pragma unroll
                    for (int e = 0; e < 8; ++e) x8[e] = ffma2(u2, k8[e], fmul2(a2, x8[e]));
                };
                int t = t0;
                for (; t + 16 <= t1; t += 16) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) step(t + i);
                }
                for (; t < t1; ++t) step(t);
                float* sr = seg + (warp * 32 + lane) * 16;
#pragma unroll
                for (int e = 0; e < 8; e += 2)
                    *reinterpret_cast<float4*>(sr + 2 * e) = make_float4(x8[e].x, x8[e].y, x8[e + 1].x, x8[e + 1].y);
            }
            __syncthreads();

            // ---- P2b: compose the segments in scan order: G <- G P_s + Q_s ---------------------
            {
                const int r = tid >> 4, cc = tid & 15;
                float gv;
                int s0;
                if (j == 0) {  // G enters the chunk as I:  G = P_0 + Q_0
                    gv = seg[r * 16 + cc] + seg[(16 + r) * 16 + cc];
                    s0 = 1;
                } else {
                    gv = gb[r * 16 + cc];  // carried from the previous pass (buffer 0)
                    s0 = 0;
                }
                int ph = 1;
                for (int s = s0; s < nseg; ++s) {
                    float* gcur = gb + ph * 256;
                    gcur[r * 16 + cc] = gv;
                    __syncthreads();
                    const float* ps = seg + s * 32 * 16;
                    float acc = ps[(16 + r) * 16 + cc];
#pragma unroll
                    for (int k = 0; k < 16; ++k) acc = fmaf(gcur[r * 16 + k], ps[k * 16 + cc], acc);
                    gv = acc;
                    ph ^= 1;
                }
                __syncthreads();  // every read of the G buffers is done
                gb[r * 16 + cc] = gv;  // G after this pass, in buffer 0
                __syncthreads();
            }
        }
        if (aborted || c + 1 == ci.nchunks) continue;

        // ---- P3: S <- S G (fp32), new operand parts for the next chunk's projections ----------
        {
            const int r = tid >> 4, cc = tid & 15;
            float nv[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int rr = r + 16 * m;
                float acc = 0.f;
                if (rr < 50) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) acc = fmaf(s32[rr * 16 + k], gb[k * 16 + cc], acc);
                }
                nv[m] = acc;
            }
            __syncthreads();  // every read of the old state is done
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int rr = r + 16 * m;
                if (rr < 50) {
                    s32[rr * 16 + cc] = nv[m];
                    put_parts(bop, rr < 16 ? 0 : 1, rr, cc, nv[m]);
                }
            }
            tcu::fence_proxy_async_smem();
            __syncthreads();
        }
    }

    // ---- tear-down: no copy in flight, TMEM released ----------------------------------------
    if (tid == 0) {  // after an abort: let copies still in flight land before the CTA exits
        for (int b = 0; b < 2; ++b)
            if (tma_pending[b]) tcu::mbar_wait(&bars[b], tma_parity[b], kWaitNs);
    }
    tcu::tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tcu::tc_fence_after_sync();
        tcu::tmem_dealloc(tmem, kTmemCols);
    }
}

// out (or fin) = ((p0 + p1) + p2) + p3 (+ addend): the four scans' planes in a fixed order.
template <typename AT>
__global__ void tc_fold_kernel(const ScanParams p) {
    const int64_t per_image = (int64_t)p.L * p.C / 4;
    const int64_t total = per_image * p.B;
    const int64_t ps = (int64_t)p.B * p.ob;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / per_image, off = (i - b * per_image) * 4;
        const int64_t o = b * p.ob + off;
        const float4 a = *reinterpret_cast<const float4*>(p.out + o);
        const float4 c1 = *reinterpret_cast<const float4*>(p.aux + o);
        const float4 c2 = *reinterpret_cast<const float4*>(p.aux + ps + o);
        const float4 c3 = *reinterpret_cast<const float4*>(p.aux + 2 * ps + o);
        float4 s = make_float4(((a.x + c1.x) + c2.x) + c3.x, ((a.y + c1.y) + c2.y) + c3.y,
                               ((a.z + c1.z) + c2.z) + c3.z, ((a.w + c1.w) + c2.w) + c3.w);
        if (p.addend) {
            const float4 e = load4(static_cast<const AT*>(p.addend) + b * p.ab + off);
            s = make_float4(s.x + e.x, s.y + e.y, s.z + e.z, s.w + e.w);
        }
        if (!p.fin) *reinterpret_cast<float4*>(p.out + o) = s;
        else if (p.fin_dtype == VH_F32) store4(static_cast<float*>(p.fin) + b * p.fb + off, s);
        else if (p.fin_dtype == VH_BF16) store4(static_cast<__nv_bfloat16*>(p.fin) + b * p.fb + off, s);
        else store4(static_cast<__half*>(p.fin) + b * p.fb + off, s);
    }
}

// ---- host side -------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// bf16 tensor map with a 16-channel x `box_tokens` box in the 32-byte swizzle; `dims` and
// `strides` (bytes, dims 1..rank-1) describe the tensor, dims[0] being its channel extent.
bool make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
              const cuuint32_t* box) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int NST, bool kSpatial>
int launch_tc(const ScanParams& p, const TcGeom& g, const TcMaps& maps, int grid, cudaStream_t st) {
    using S = TcSmem<NST>;
    const void* fn = reinterpret_cast<const void*>(&srnl_tc_kernel<NST, kSpatial>);
    if (!ensure_smem_attr(fn, S::kLaunch))
        return fail(VH_E_DEVICE, "srnl tc scan: cannot reserve %zu bytes of shared memory", S::kLaunch);
    srnl_tc_kernel<NST, kSpatial><<<grid, kThreads, S::kLaunch, st>>>(p, g, maps);
    return launch_status("srnl tc scan");
}

template <bool kSpatial>
int launch_tc_nst(const ScanParams& p, const TcGeom& g, const TcMaps& maps, int grid, int max_chunk, cudaStream_t st) {
    if (max_chunk <= kST) return launch_tc<1, kSpatial>(p, g, maps, grid, st);
    if (max_chunk <= 2 * kST) return launch_tc<2, kSpatial>(p, g, maps, grid, st);
    return launch_tc<4, kSpatial>(p, g, maps, grid, st);
}

inline int box_for(int chunk, int extent) { return std::max(1, std::min(std::min(chunk, kBoxMax), extent)); }

}  // namespace tc

// The tensor-core scan applies to head_dim 16 with bf16 x and raw bf16 queries, in the image
// layout (channels-last rows), the serialized-scans layout with 16-channel heads, and packed
// sequences; the spatial operator also needs the three aux planes.
bool tc_applicable(const ScanParams& p, bool spatial) {
    if (p.q_mode != 0) return false;
    if (!tc::encode_fn()) return false;
    const int esz = 2;
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    if (!al16(p.x) || !al16(p.q)) return false;
    if (spatial) {
        if (!p.aux) return false;
        if (p.xh != 16 || p.qh != 16) return false;
        if ((p.xt * esz) % 16 || (p.qt * esz) % 16 || (p.xb * esz) % 16 || (p.qb * esz) % 16) return false;
        if (!p.remap && ((p.xd * esz) % 16 || (p.qd * esz) % 16)) return false;
        if ((p.ob % 4) || (reinterpret_cast<uintptr_t>(p.out) & 15) || (reinterpret_cast<uintptr_t>(p.aux) & 15))
            return false;
        return true;
    }
    return (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
}

int run_tc_spatial(const ScanParams& p, int io_dtype, cudaStream_t st) {
    using namespace tc;
    TcMaps maps{};
    TcGeom g{};
    const int C = p.C;
    if (p.remap) {
        g.layout = 0;
        g.box_rows = box_for(p.W, p.W);
        g.box_cols = box_for(p.H, p.H);
        const cuuint64_t xd[4] = {(cuuint64_t)C, (cuuint64_t)p.W, (cuuint64_t)p.H, (cuuint64_t)p.B};
        const cuuint64_t xs[3] = {(cuuint64_t)p.xt * 2, (cuuint64_t)p.W * p.xt * 2, (cuuint64_t)p.xb * 2};
        const cuuint64_t qs[3] = {(cuuint64_t)p.qt * 2, (cuuint64_t)p.W * p.qt * 2, (cuuint64_t)p.qb * 2};
        const cuuint32_t br[4] = {16, (cuuint32_t)g.box_rows, 1, 1};
        const cuuint32_t bc[4] = {16, 1, (cuuint32_t)g.box_cols, 1};
        if (!make_map(&maps.x[0], p.x, 4, xd, xs, br) || !make_map(&maps.q[0], p.q, 4, xd, qs, br) ||
            !make_map(&maps.x[1], p.x, 4, xd, xs, bc) || !make_map(&maps.q[1], p.q, 4, xd, qs, bc))
            return fail(VH_E_DEVICE, "srnl tc scan: tensor map encoding failed");
    } else {
        g.layout = 1;
        g.box_rows = g.box_cols = box_for(std::max(p.W, p.H), p.L);
        // rows use chunks of W, columns chunks of H: one box size serves both when it covers
        // the longer one in at most two boxes per pass
        const cuuint64_t d[4] = {(cuuint64_t)C, (cuuint64_t)p.L, 4, (cuuint64_t)p.B};
        const cuuint64_t xs[3] = {(cuuint64_t)p.xt * 2, (cuuint64_t)p.xd * 2, (cuuint64_t)p.xb * 2};
        const cuuint64_t qs[3] = {(cuuint64_t)p.qt * 2, (cuuint64_t)p.qd * 2, (cuuint64_t)p.qb * 2};
        const cuuint32_t b[4] = {16, (cuuint32_t)g.box_rows, 1, 1};
        if (!make_map(&maps.x[0], p.x, 4, d, xs, b) || !make_map(&maps.q[0], p.q, 4, d, qs, b))
            return fail(VH_E_DEVICE, "srnl tc scan: tensor map encoding failed");
        maps.x[1] = maps.x[0];
        maps.q[1] = maps.q[0];
    }
    const int grid = p.B * p.heads * 4;
    int rc = launch_tc_nst<true>(p, g, maps, grid, std::max(p.W, p.H), st);
    if (rc) return rc;
    const int64_t total = (int64_t)p.B * p.L * p.C / 4;
    const int fgrid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
    switch (io_dtype) {
        case VH_F32: tc_fold_kernel<float><<<fgrid, 256, 0, st>>>(p); break;
        case VH_F16: tc_fold_kernel<__half><<<fgrid, 256, 0, st>>>(p); break;
        default: tc_fold_kernel<__nv_bfloat16><<<fgrid, 256, 0, st>>>(p);
    }
    return launch_status("srnl tc fold");
}

int run_tc_sequence(const ScanParams& p, cudaStream_t st) {
    using namespace tc;
    TcMaps maps{};
    TcGeom g{};
    g.layout = 2;
    int maxc = 1;
    for (int r = 0; r < p.R; ++r) maxc = std::max(maxc, p.chunk[r]);
    g.box_rows = g.box_cols = box_for(maxc, p.L);
    const int chains = p.B * p.R * p.heads;
    const cuuint64_t xd[3] = {16, (cuuint64_t)p.L, (cuuint64_t)chains};
    const cuuint64_t xs[2] = {32, (cuuint64_t)p.L * 32};
    const cuuint64_t qd[3] = {(cuuint64_t)p.C, (cuuint64_t)p.L, (cuuint64_t)p.B * p.R};
    const cuuint64_t qs[2] = {(cuuint64_t)p.C * 2, (cuuint64_t)p.L * p.C * 2};
    const cuuint32_t b[3] = {16, (cuuint32_t)g.box_rows, 1};
    if (!make_map(&maps.x[0], p.x, 3, xd, xs, b) || !make_map(&maps.q[0], p.q, 3, qd, qs, b))
        return fail(VH_E_DEVICE, "srnl tc scan: tensor map encoding failed");
    maps.x[1] = maps.x[0];
    maps.q[1] = maps.q[0];
    return launch_tc_nst<false>(p, g, maps, chains, maxc, st);
}

}  // namespace vh

extern "C" int vh_tc_status(int32_t reset) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, vh::tc::g_tc_status, sizeof(v)) != cudaSuccess) return -1;
    if (reset) {
        const unsigned int z = 0;
        cudaMemcpyToSymbol(vh::tc::g_tc_status, &z, sizeof(z));
    }
    return (int)v;
}
