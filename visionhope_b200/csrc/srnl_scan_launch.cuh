// Host-side launch templates of the SRNL scans.  Included only by the per-head-dim
// translation units (srnl_scan_d*.cu), which instantiate them explicitly so the five
// head dims compile in parallel.
#pragma once

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "abi_util.h"
#include "srnl_scan.cuh"
#include "srnl_warp.cuh"

namespace vh {

struct ScanPlan {
    int tile, nch;
};

// Tile = tokens of one chunk staged per step (power of two, 4..64); nch = chains per CTA
// such that both the token-parallel phase (nch * tile threads) and the gain recurrence
// (nch * D threads) fit in one 128-thread CTA.
inline ScanPlan plan_scan(int D, int max_chunk, bool spatial) {
    int tile = 4;
    while (tile < max_chunk && tile < 64) tile *= 2;
    int nch = std::min(kScanThreads / D, kScanThreads / tile);
    nch = std::min(nch, 8);
    if (spatial) nch = std::max(2, nch & ~1);
    return {tile, nch};
}

template <int D, typename XT, typename QT, int KIND, bool MMA>
size_t scan_smem(const ScanPlan& pl) {
    return ScanSmem<D>(pl.nch, pl.tile, MMA).total;
}

// The tensor-core token phase applies to D = 16 with bf16 x and raw bf16 queries.
template <int D, typename XT, typename QT>
constexpr bool mma_capable() {
    return D == 16 && std::is_same<XT, __nv_bfloat16>::value && std::is_same<QT, __nv_bfloat16>::value;
}

// Halve the token tile (raising chains per CTA only within the thread budget) until the
// shared-memory carve-up fits under `limit`; the tensor-core variant aims at <= 56 KB so
// four CTAs (the register-file limit) share an SM.
template <int D, typename XT, typename QT, int KIND, bool MMA>
ScanPlan fit_plan(int max_chunk) {
    const size_t limit = MMA ? 56 * 1024 : 200 * 1024;
    const bool spatial = KIND != kKindSeq;
    ScanPlan pl = plan_scan(D, max_chunk, spatial);
    while (scan_smem<D, XT, QT, KIND, MMA>(pl) > limit && pl.tile > (MMA ? 16 : 4)) {
        pl.tile /= 2;
        const int nch = std::min(std::min(kScanThreads / D, kScanThreads / pl.tile), pl.nch);
        pl.nch = spatial ? std::max(2, nch & ~1) : nch;
    }
    while (scan_smem<D, XT, QT, KIND, MMA>(pl) > limit && pl.nch > (spatial ? 2 : 1)) pl.nch -= spatial ? 2 : 1;
    return pl;
}

template <int D, typename XT, typename QT, int KIND, bool MMA>
int launch_scan(ScanParams p, const ScanPlan& pl, dim3 grid, cudaStream_t st) {
    p.nch = pl.nch;
    p.tile = pl.tile;
    p.log2tile = 0;
    while ((1 << p.log2tile) < pl.tile) ++p.log2tile;
    p.kind = KIND;
    const size_t smem = scan_smem<D, XT, QT, KIND, MMA>(pl);
    const void* fn = reinterpret_cast<const void*>(&srnl_scan_kernel<D, XT, QT, KIND, MMA>);
    if (!ensure_smem_attr(fn, smem))
        return fail(VH_E_DEVICE, "srnl scan: cannot reserve %zu bytes of shared memory", smem);
    srnl_scan_kernel<D, XT, QT, KIND, MMA><<<grid, kScanThreads, smem, st>>>(p);
    return launch_status("srnl scan");
}

// Warp-per-chain scan (D = 16, bf16), four warps per CTA: the four scans of one (b, head)
// (kKindBoth, needs the three aux planes) or four sequence chains (kKindSeq).
template <int KIND, int TILE>
int launch_warp_tile(ScanParams p, int pairs_or_chains, cudaStream_t st) {
    p.kind = KIND;
    p.nch = wpc::kWarps;
    p.tile = TILE;
    p.log2tile = TILE == 16 ? 4 : 5;
    const size_t smem = sizeof(wpc::ChainSmemT<TILE>) * wpc::kWarps;
    const int per_cta = KIND == kKindBoth ? 1 : wpc::kWarps;
    const dim3 grid((pairs_or_chains + per_cta - 1) / per_cta, KIND == kKindSeq ? p.R : 1);
    const void* fn = reinterpret_cast<const void*>(&wpc::srnl_warp_kernel<KIND, TILE>);
    if (!ensure_smem_attr(fn, smem))
        return fail(VH_E_DEVICE, "srnl warp scan: cannot reserve %zu bytes of shared memory", smem);
    wpc::srnl_warp_kernel<KIND, TILE><<<grid, wpc::kThreads, smem, st>>>(p);
    return launch_status("srnl warp scan");
}

// Steps of 16 tokens when no chunk is longer (VisionHOPE stages 3 and 4), else of 32.
template <int KIND>
int launch_warp(const ScanParams& p, int pairs_or_chains, cudaStream_t st) {
    int maxc = 0;
    if (KIND == kKindSeq) {
        for (int r = 0; r < p.R; ++r) maxc = std::max(maxc, p.chunk[r]);
    } else {
        maxc = std::max(p.H, p.W);
    }
    return maxc <= 16 ? launch_warp_tile<KIND, 16>(p, pairs_or_chains, st)
                      : launch_warp_tile<KIND, 32>(p, pairs_or_chains, st);
}

// Sequences: the warp-per-chain scan when it applies (D = 16, bf16, chunks of 9+ tokens).
// Spatial passes without the aux planes: the CTA-lockstep scan, with its tensor-core token
// phase where it applies.
template <int D, typename XT, typename QT, int KIND>
int launch_auto(const ScanParams& p, int max_chunk, int pairs_or_chains, cudaStream_t st) {
    const bool spatial = KIND != kKindSeq;
    if constexpr (mma_capable<D, XT, QT>()) {
        if (max_chunk > 8) {
            if (!spatial) return launch_warp<kKindSeq>(p, pairs_or_chains, st);
            const ScanPlan pl = fit_plan<D, XT, QT, KIND, true>(max_chunk);
            dim3 grid((pairs_or_chains + pl.nch / 2 - 1) / (pl.nch / 2), 1);
            return launch_scan<D, XT, QT, KIND, true>(p, pl, grid, st);
        }
    }
    const ScanPlan pl = fit_plan<D, XT, QT, KIND, false>(max_chunk);
    const int per_cta = spatial ? pl.nch / 2 : pl.nch;
    dim3 grid((pairs_or_chains + per_cta - 1) / per_cta, spatial ? 1 : p.R);
    return launch_scan<D, XT, QT, KIND, false>(p, pl, grid, st);
}

// Writes (final dtype)(out + addend) when the scans ran without folding it in (srnl_scan.cu).
int launch_spatial_finalize(const ScanParams& p, int io_dtype, cudaStream_t st);

// The chunk-parallel tensor-core scan (srnl_tc.cu).
bool tc_applicable(const ScanParams& p, bool spatial);
int run_tc_spatial(const ScanParams& p, int io_dtype, cudaStream_t st);
int run_tc_sequence(const ScanParams& p, cudaStream_t st);

// Which D = 16 bf16 scan runs.  The chunk-parallel tensor-core scan gives each chain a whole
// CTA (two per SM for chunks of up to 256 tokens, one above) and runs a chunk's tokens in
// parallel, at a fixed cost per chunk; the warp-per-chain scan runs one token after the other
// and wins when chains are plentiful or chunks short.  Measured on B200 (bf16, image layout,
// tensor-core against warp scan, ms):
//   chunks of 56+ tokens: 24 chains of 128 x 512 2.28 / 6.46; 64, 128 and 256 chains of
//     56 x 56 0.21 / 0.32, 0.21 / 0.33, 0.27 / 0.33; 112 chains of 32 x 128 0.41 / 0.42;
//     160 chains of 16 x 64 0.218 / 0.220;
//   chunks of 14 and 28 tokens: 128 chains of 14 x 14 0.056 / 0.040, 256 chains of 28 x 28
//     0.122 / 0.097; 2048+ chains at every VisionHOPE-T stage, several times slower.
// So the tensor-core scan runs for chunks of 48+ tokens while every chain has a CTA slot in the
// first wave, and for shorter chunks only up to a third of an SM per chain.  VH_SRNL_SCAN=tc or
// =warp forces one of them (where it applies).
inline bool use_tc_scan(const ScanParams& p, bool spatial, int chains, int max_chunk) {
    const char* env = std::getenv("VH_SRNL_SCAN");
    if (env && std::strcmp(env, "warp") == 0) return false;
    if (!tc_applicable(p, spatial)) return false;
    if (env && std::strcmp(env, "tc") == 0) return true;
    const int sms = sm_count();
    if (max_chunk >= 48) return chains <= (max_chunk > 256 ? 1 : 2) * sms;
    return 3 * chains <= sms;
}

template <int D, typename T>
int run_spatial(const ScanParams& p, cudaStream_t st) {
    const int pairs = p.B * p.heads;
    if constexpr (mma_capable<D, T, T>()) {
        if (use_tc_scan(p, true, 4 * pairs, std::max(p.H, p.W))) return run_tc_spatial(p, VH_BF16, st);
        if (p.aux) return launch_warp<kKindBoth>(p, pairs, st);
    }
    int rc = launch_auto<D, T, T, kKindRows>(p, p.W, pairs, st);
    if (rc) return rc;
    rc = launch_auto<D, T, T, kKindCols>(p, p.H, pairs, st);
    if (rc || !p.fin) return rc;
    const int io = std::is_same<T, float>::value ? VH_F32 : std::is_same<T, __half>::value ? VH_F16 : VH_BF16;
    return launch_spatial_finalize(p, io, st);
}

template <int D, typename XT, typename QT>
int run_sequence(const ScanParams& p, cudaStream_t st) {
    int maxc = 1;
    for (int r = 0; r < p.R; ++r) maxc = std::max(maxc, p.chunk[r]);
    if constexpr (mma_capable<D, XT, QT>()) {
        if (use_tc_scan(p, false, p.B * p.R * p.heads, maxc)) return run_tc_sequence(p, st);
    }
    return launch_auto<D, XT, QT, kKindSeq>(p, maxc, p.B * p.heads, st);
}

template <int D, typename XT, typename QT, int KIND>
void set_attr_one() {
    // Reserve the opt-in maximum once per device; every launch re-checks its own size.
    ensure_smem_attr(reinterpret_cast<const void*>(&srnl_scan_kernel<D, XT, QT, KIND, false>), 48 * 1024 + 1);
    if constexpr (mma_capable<D, XT, QT>())
        ensure_smem_attr(reinterpret_cast<const void*>(&srnl_scan_kernel<D, XT, QT, KIND, true>), 48 * 1024 + 1);
}

template <int D>
void set_attr_d() {
    set_attr_one<D, float, float, kKindRows>();
    set_attr_one<D, float, float, kKindCols>();
    set_attr_one<D, __nv_bfloat16, __nv_bfloat16, kKindRows>();
    set_attr_one<D, __nv_bfloat16, __nv_bfloat16, kKindCols>();
    set_attr_one<D, __half, __half, kKindRows>();
    set_attr_one<D, __half, __half, kKindCols>();
    set_attr_one<D, float, float, kKindSeq>();
    set_attr_one<D, __nv_bfloat16, __nv_bfloat16, kKindSeq>();
    set_attr_one<D, __half, __half, kKindSeq>();
    set_attr_one<D, __nv_bfloat16, float, kKindSeq>();
    set_attr_one<D, __half, float, kKindSeq>();
}

#define VH_INSTANTIATE_SCAN(D)                                                              \
    template int run_spatial<D, float>(const ScanParams&, cudaStream_t);                      \
    template int run_spatial<D, __nv_bfloat16>(const ScanParams&, cudaStream_t);              \
    template int run_spatial<D, __half>(const ScanParams&, cudaStream_t);                     \
    template int run_sequence<D, float, float>(const ScanParams&, cudaStream_t);              \
    template int run_sequence<D, __nv_bfloat16, __nv_bfloat16>(const ScanParams&, cudaStream_t); \
    template int run_sequence<D, __half, __half>(const ScanParams&, cudaStream_t);            \
    template int run_sequence<D, __nv_bfloat16, float>(const ScanParams&, cudaStream_t);      \
    template int run_sequence<D, __half, float>(const ScanParams&, cudaStream_t);             \
    template void set_attr_d<D>();

}  // namespace vh
