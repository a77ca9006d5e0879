// Host-side helpers shared by the libvhope entry points: thread-local error text,
// validation shorthands and launch-status translation.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include "vhope.h"

namespace vh {

// Records a printf-style message as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears this thread's last error.
void clear_error();
// Translates the launch status of the most recent kernel launch: 0 or a positive cudaError_t.
int launch_status(const char* what);

inline size_t dtype_size(int dt) { return dt == VH_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == VH_F32 || dt == VH_BF16 || dt == VH_F16; }
inline bool head_dim_ok(int d) { return d == 4 || d == 8 || d == 16 || d == 32 || d == 64; }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Sets the dynamic shared-memory limit of a kernel once per device; returns false on failure.
bool ensure_smem_attr(const void* func, size_t bytes);

// Number of SMs of the current device (looked up once per device; 148 if the query fails).
int sm_count();

}  // namespace vh
