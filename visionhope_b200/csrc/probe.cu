// Measurement helper: an FFMA throughput probe used by bench.py to measure the FP32
// (non-tensor) peak of the device, the denominator of the SRNL scan's roofline.
#include "abi_util.h"
#include "common.cuh"

namespace vh {

// 8 independent FMA chains per thread, `iters` rounds; the result is stored so the work
// cannot be eliminated.  FLOPs = 2 * 8 * 4 * iters * threads.
__global__ void __launch_bounds__(256) ffma_probe_kernel(float* out, int iters, float a, float b) {
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = fmaf(r[i], a, b);
        }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += r[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace vh

extern "C" int vh_probe_ffma(float* out, int32_t blocks, int32_t iters, vh_stream_t stream) {
    vh::clear_error();
    if (!out || blocks <= 0 || iters <= 0) return vh::fail(VH_E_ARG, "vh_probe_ffma: bad arguments");
    vh::ffma_probe_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(out, iters, 0.9999f, 1e-4f);
    return vh::launch_status("ffma probe");
}
