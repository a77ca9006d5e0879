// libvhope: library-wide entry points (init, error text, version) and host helpers.
#include <atomic>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <set>
#include <utility>

#include "abi_util.h"
#include "vhope.h"

namespace vh {

namespace {
thread_local char g_last_error[512] = {0};
thread_local int g_launches = 0;
std::mutex g_attr_mu;
std::set<std::pair<int, const void*>>& attr_done() {
    static std::set<std::pair<int, const void*>> s;
    return s;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() {
    g_last_error[0] = 0;
    g_launches = 0;
}

int launch_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail((int)e, "%s: launch failed: %s", what, cudaGetErrorString(e));
    ++g_launches;
    return 0;
}

bool ensure_smem_attr(const void* func, size_t bytes) {
    if (bytes <= 48 * 1024) return true;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    auto key = std::make_pair(dev, func);
    if (attr_done().count(key)) return true;
    // Always request the per-block maximum so later calls with larger tiles need no change.
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return false;
    if ((size_t)optin < bytes) return false;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess)
        return false;
    attr_done().insert(key);
    return true;
}

int sm_count() {
    // Per device; concurrent first calls may both query the count and store the same value.
    static std::atomic<int> counts[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = counts[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Defined in the kernel translation units: set every kernel's attributes for `device`.
int init_scan_kernels();
int init_norm_kernels();
int init_dw_kernels();

}  // namespace vh

extern "C" int vh_init(int32_t device) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return vh::fail(VH_E_DEVICE, "vh_init: no CUDA device");
    if (cudaSetDevice(device) != cudaSuccess)
        return vh::fail(VH_E_DEVICE, "vh_init: cannot select device %d", device);
    int rc = vh::init_scan_kernels();
    if (rc == 0) rc = vh::init_norm_kernels();
    if (rc == 0) rc = vh::init_dw_kernels();
    cudaSetDevice(prev);
    return rc;
}

extern "C" const char* vh_last_error(void) { return vh::g_last_error; }

extern "C" int vh_last_launch_count(void) { return vh::g_launches; }

extern "C" const char* vh_version(void) { return "vhope-b200 0.1 (sm_100a)"; }
