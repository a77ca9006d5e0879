// Host-side launch templates of the SRNL scans.  Included only by the per-head-dim
// translation units (srnl_scan_d*.cu), which instantiate them explicitly so the five
// head dims compile in parallel.
#pragma once

#include <algorithm>

#include "abi_util.h"
#include "srnl_scan.cuh"

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

template <int D, typename XT, typename QT, int KIND>
size_t scan_smem(const ScanPlan& pl) {
    return ScanSmem<D>(pl.nch, pl.tile).total;
}

// Halve the token tile (raising chains per CTA only within the thread budget) until the
// shared-memory carve-up fits comfortably under the 227 KB per-CTA limit.
template <int D, typename XT, typename QT, int KIND>
ScanPlan fit_plan(int max_chunk) {
    constexpr size_t kLimit = 200 * 1024;
    ScanPlan pl = plan_scan(D, max_chunk, KIND != kKindSeq);
    while (scan_smem<D, XT, QT, KIND>(pl) > kLimit && pl.tile > 4) {
        pl.tile /= 2;
        const int nch = std::min(std::min(kScanThreads / D, kScanThreads / pl.tile), pl.nch);
        pl.nch = KIND != kKindSeq ? std::max(2, nch & ~1) : nch;
    }
    while (scan_smem<D, XT, QT, KIND>(pl) > kLimit && pl.nch > (KIND != kKindSeq ? 2 : 1))
        pl.nch -= KIND != kKindSeq ? 2 : 1;
    return pl;
}

template <int D, typename XT, typename QT, int KIND>
int launch_scan(ScanParams p, const ScanPlan& pl, dim3 grid, cudaStream_t st) {
    p.nch = pl.nch;
    p.tile = pl.tile;
    p.log2tile = 0;
    while ((1 << p.log2tile) < pl.tile) ++p.log2tile;
    p.kind = KIND;
    const size_t smem = scan_smem<D, XT, QT, KIND>(pl);
    const void* fn = reinterpret_cast<const void*>(&srnl_scan_kernel<D, XT, QT, KIND>);
    if (!ensure_smem_attr(fn, smem))
        return fail(VH_E_DEVICE, "srnl scan: cannot reserve %zu bytes of shared memory", smem);
    srnl_scan_kernel<D, XT, QT, KIND><<<grid, kScanThreads, smem, st>>>(p);
    return launch_status("srnl scan");
}

template <int D, typename T>
int run_spatial(const ScanParams& p, cudaStream_t st) {
    const ScanPlan rows = fit_plan<D, T, T, kKindRows>(p.W), cols = fit_plan<D, T, T, kKindCols>(p.H);
    const int pairs = p.B * p.heads;
    dim3 grow((pairs + rows.nch / 2 - 1) / (rows.nch / 2)), gcol((pairs + cols.nch / 2 - 1) / (cols.nch / 2));
    int rc = launch_scan<D, T, T, kKindRows>(p, rows, grow, st);
    if (rc) return rc;
    return launch_scan<D, T, T, kKindCols>(p, cols, gcol, st);
}

template <int D, typename XT, typename QT>
int run_sequence(const ScanParams& p, cudaStream_t st) {
    int maxc = 1;
    for (int r = 0; r < p.R; ++r) maxc = std::max(maxc, p.chunk[r]);
    const ScanPlan pl = fit_plan<D, XT, QT, kKindSeq>(maxc);
    dim3 grid((p.B * p.heads + pl.nch - 1) / pl.nch, p.R);
    return launch_scan<D, XT, QT, kKindSeq>(p, pl, grid, st);
}

template <int D, typename XT, typename QT, int KIND>
void set_attr_one() {
    // Reserve the opt-in maximum once per device; every launch re-checks its own size.
    ensure_smem_attr(reinterpret_cast<const void*>(&srnl_scan_kernel<D, XT, QT, KIND>), 48 * 1024 + 1);
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
