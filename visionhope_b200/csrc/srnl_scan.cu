// Host launchers and C entry points of the SRNL scans (spatial operator and packed sequences).
#include <algorithm>

#include "abi_util.h"
#include "srnl_scan.cuh"

namespace vh {

// Explicitly instantiated in srnl_scan_d{4,8,16,32,64}.cu.
template <int D, typename T> int run_spatial(const ScanParams& p, cudaStream_t st);
template <int D, typename XT, typename QT> int run_sequence(const ScanParams& p, cudaStream_t st);
template <int D> void set_attr_d();

namespace {

template <typename T>
int spatial_dispatch_d(int D, const ScanParams& p, cudaStream_t st) {
    switch (D) {
        case 4: return run_spatial<4, T>(p, st);
        case 8: return run_spatial<8, T>(p, st);
        case 16: return run_spatial<16, T>(p, st);
        case 32: return run_spatial<32, T>(p, st);
        case 64: return run_spatial<64, T>(p, st);
    }
    return fail(VH_E_HEADDIM, "unsupported head_dim %d", D);
}

template <typename XT, typename QT>
int sequence_dispatch_d(int D, const ScanParams& p, cudaStream_t st) {
    switch (D) {
        case 4: return run_sequence<4, XT, QT>(p, st);
        case 8: return run_sequence<8, XT, QT>(p, st);
        case 16: return run_sequence<16, XT, QT>(p, st);
        case 32: return run_sequence<32, XT, QT>(p, st);
        case 64: return run_sequence<64, XT, QT>(p, st);
    }
    return fail(VH_E_HEADDIM, "unsupported head_dim %d", D);
}

SrnlConsts to_consts(const vh_srnl_consts& c) {
    return {c.step_scale, c.min_retention, c.retention_bias, c.injection_margin,
            c.spectral_factor, c.spectral_clamp};
}

bool consts_ok(const vh_srnl_consts& c) {
    return c.step_scale > 0.f && c.min_retention >= 0.f && c.min_retention < 1.f &&
           c.injection_margin > 0.f && c.injection_margin < 1.f && c.spectral_factor > 0.f;
}

// Vector width (bytes) of one token row copy and the element multiple every stride must keep.
int row_vec_bytes(int D, int dt) {
    const int rb = D * (int)dtype_size(dt);
    return rb < 16 ? rb : 16;
}

}  // namespace

// (final dtype)(out + addend) over [B, H*W*C] in groups of four channels.
template <typename AT>
__global__ void spatial_finalize_kernel(const float* __restrict__ out, int64_t ob,
                                        const AT* __restrict__ addend, int64_t ab, void* fin,
                                        int fdt, int64_t fb, int64_t groups_per_image, int B) {
    const int64_t total = groups_per_image * B;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / groups_per_image, r = (i - b * groups_per_image) * 4;
        float4 v = load4(out + b * ob + r);
        if (addend) {
            const float4 e = load4(addend + b * ab + r);
            v = make_float4(v.x + e.x, v.y + e.y, v.z + e.z, v.w + e.w);
        }
        if (fdt == VH_F32) store4(static_cast<float*>(fin) + b * fb + r, v);
        else if (fdt == VH_BF16) store4(static_cast<__nv_bfloat16*>(fin) + b * fb + r, v);
        else store4(static_cast<__half*>(fin) + b * fb + r, v);
    }
}

int launch_spatial_finalize(const ScanParams& p, int io_dtype, cudaStream_t st) {
    const int64_t groups = (int64_t)p.L * p.C / 4, total = groups * p.B;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
    switch (io_dtype) {
        case VH_F32:
            spatial_finalize_kernel<float><<<grid, 256, 0, st>>>(p.out, p.ob, static_cast<const float*>(p.addend),
                                                                 p.ab, p.fin, p.fin_dtype, p.fb, groups, p.B);
            break;
        case VH_BF16:
            spatial_finalize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
                p.out, p.ob, static_cast<const __nv_bfloat16*>(p.addend), p.ab, p.fin, p.fin_dtype, p.fb, groups, p.B);
            break;
        default:
            spatial_finalize_kernel<__half><<<grid, 256, 0, st>>>(p.out, p.ob, static_cast<const __half*>(p.addend),
                                                                  p.ab, p.fin, p.fin_dtype, p.fb, groups, p.B);
    }
    return launch_status("srnl spatial finalize");
}

int init_scan_kernels() {
    set_attr_d<4>();
    set_attr_d<8>();
    set_attr_d<16>();
    set_attr_d<32>();
    set_attr_d<64>();
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(VH_E_DEVICE, "vh_init: %s", cudaGetErrorString(e));
    return 0;
}

}  // namespace vh

using namespace vh;

extern "C" int vh_srnl_spatial_fwd(const vh_srnl_spatial_args* a, vh_stream_t stream) {
    clear_error();
    if (!a) return fail(VH_E_ARG, "vh_srnl_spatial_fwd: null args");
    if (!a->mem.m || !a->mem.v || !a->mem.k || !a->mem.eta || !a->mem.alpha || !a->x || !a->q ||
        !a->skip || !a->weight || !a->out)
        return fail(VH_E_ARG, "vh_srnl_spatial_fwd: null pointer argument");
    if (!dtype_ok(a->io_dtype)) return fail(VH_E_DTYPE, "vh_srnl_spatial_fwd: bad io dtype");
    if (!head_dim_ok(a->head_dim))
        return fail(VH_E_HEADDIM, "SRNL head_dim must be one of 4, 8, 16, 32, 64 (got %d)", a->head_dim);
    if (a->batch <= 0 || a->height <= 0 || a->width <= 0 || a->heads <= 0)
        return fail(VH_E_SHAPE, "vh_srnl_spatial_fwd: batch, height, width and heads must be positive");
    if (!consts_ok(a->consts)) return fail(VH_E_ARG, "vh_srnl_spatial_fwd: invalid recurrence constants");
    const int64_t L = (int64_t)a->height * a->width;
    const int64_t C = (int64_t)a->heads * a->head_dim;
    if (L > (int64_t)1 << 30 || (int64_t)a->batch * a->heads > (int64_t)1 << 30)
        return fail(VH_E_RANGE, "vh_srnl_spatial_fwd: sizes exceed the supported range");
    const int vb = row_vec_bytes(a->head_dim, a->io_dtype);
    const int64_t ve = vb / (int64_t)dtype_size(a->io_dtype);
    if (!aligned(a->x, vb) || !aligned(a->q, vb) || a->x_batch_stride % ve || a->q_batch_stride % ve ||
        a->x_token_stride % ve || a->q_token_stride % ve || a->x_head_stride % ve ||
        a->q_head_stride % ve || (!a->remap && (a->x_dir_stride % ve || a->q_dir_stride % ve)))
        return fail(VH_E_ALIGN, "vh_srnl_spatial_fwd: x/q pointers or strides not %d-byte aligned", vb);
    if (!aligned(a->out, 16) || a->out_batch_stride % 4)
        return fail(VH_E_ALIGN, "vh_srnl_spatial_fwd: out must be 16-byte aligned");
    if (a->x_token_stride < a->head_dim || a->q_token_stride < a->head_dim ||
        a->x_head_stride < a->head_dim || a->q_head_stride < a->head_dim ||
        a->out_batch_stride < L * C)
        return fail(VH_E_SHAPE, "vh_srnl_spatial_fwd: token/head strides smaller than head_dim");
    if (a->aux && (a->aux == a->out || !aligned(a->aux, 16)))
        return fail(VH_E_ARG, "vh_srnl_spatial_fwd: aux must be a 16-byte aligned plane distinct from out");
    if (a->addend && !a->final_out)
        return fail(VH_E_ARG, "vh_srnl_spatial_fwd: addend requires final_out");
    if (a->final_out) {
        if (!dtype_ok(a->final_dtype)) return fail(VH_E_DTYPE, "vh_srnl_spatial_fwd: bad final dtype");
        if (!aligned(a->final_out, 16) || a->final_batch_stride % 4)
            return fail(VH_E_ALIGN, "vh_srnl_spatial_fwd: final_out must be 16-byte aligned");
        if (a->final_batch_stride < L * C)
            return fail(VH_E_SHAPE, "vh_srnl_spatial_fwd: final_batch_stride smaller than H*W*C");
    }
    if (a->addend) {
        if (!aligned(a->addend, 4 * dtype_size(a->io_dtype)) || a->addend_batch_stride % 4)
            return fail(VH_E_ALIGN, "vh_srnl_spatial_fwd: addend must be aligned to 4 elements");
        if (a->addend_batch_stride < L * C)
            return fail(VH_E_SHAPE, "vh_srnl_spatial_fwd: addend_batch_stride smaller than H*W*C");
    }

    ScanParams p{};
    p.Mm = a->mem.m; p.Mv = a->mem.v; p.Mk = a->mem.k; p.Me = a->mem.eta; p.Ma = a->mem.alpha;
    p.mem_per_chain = a->mem.per_chain != 0;
    p.x = a->x; p.q = a->q;
    p.xb = a->x_batch_stride; p.xd = a->x_dir_stride; p.xt = a->x_token_stride; p.xh = a->x_head_stride;
    p.qb = a->q_batch_stride; p.qd = a->q_dir_stride; p.qt = a->q_token_stride; p.qh = a->q_head_stride;
    p.remap = a->remap != 0;
    p.q_mode = 0;
    p.out = a->out; p.ob = a->out_batch_stride;
    p.skip = a->skip; p.skip_per_dir = a->skip_per_dir != 0; p.weight = a->weight;
    p.B = a->batch; p.R = 4; p.heads = a->heads; p.L = (int)L; p.H = a->height; p.W = a->width;
    p.C = (int)C;
    p.chunk[0] = p.chunk[1] = a->width;
    p.chunk[2] = p.chunk[3] = a->height;
    p.k = to_consts(a->consts);
    p.aux = a->aux;
    p.addend = a->addend;
    p.ab = a->addend_batch_stride;
    p.fin = a->final_out;
    p.fin_dtype = a->final_dtype;
    p.fb = a->final_batch_stride;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->io_dtype) {
        case VH_F32: return spatial_dispatch_d<float>(a->head_dim, p, st);
        case VH_BF16: return spatial_dispatch_d<__nv_bfloat16>(a->head_dim, p, st);
        default: return spatial_dispatch_d<__half>(a->head_dim, p, st);
    }
}

extern "C" int vh_srnl_sequence_fwd(const vh_srnl_sequence_args* a, vh_stream_t stream) {
    clear_error();
    if (!a) return fail(VH_E_ARG, "vh_srnl_sequence_fwd: null args");
    if (!a->mem.m || !a->mem.v || !a->mem.k || !a->mem.eta || !a->mem.alpha || !a->x || !a->q || !a->y)
        return fail(VH_E_ARG, "vh_srnl_sequence_fwd: null pointer argument");
    if (!dtype_ok(a->x_dtype) || !dtype_ok(a->q_dtype))
        return fail(VH_E_DTYPE, "vh_srnl_sequence_fwd: bad dtype");
    if (a->q_mode == 0 && a->q_dtype != a->x_dtype)
        return fail(VH_E_DTYPE, "SRNL raw queries must match the input dtype");
    if (a->q_mode == 1 && a->q_dtype != VH_F32)
        return fail(VH_E_DTYPE, "SRNL normalized queries must be fp32");
    if (a->q_mode != 0 && a->q_mode != 1) return fail(VH_E_ARG, "vh_srnl_sequence_fwd: bad q_mode");
    if (!head_dim_ok(a->head_dim))
        return fail(VH_E_HEADDIM, "SRNL head_dim must be one of 4, 8, 16, 32, 64 (got %d)", a->head_dim);
    if (a->dirs != 1 && a->dirs != 2 && a->dirs != 4)
        return fail(VH_E_SHAPE, "SRNL supports 1, 2 or 4 directions (got %d)", a->dirs);
    if (a->batch <= 0 || a->heads <= 0 || a->length <= 0)
        return fail(VH_E_SHAPE, "SRNL requires nonempty batches and sequences");
    for (int r = 0; r < a->dirs; ++r)
        if (a->chunk[r] <= 0) return fail(VH_E_SHAPE, "SRNL chunk length must be positive");
    if (!consts_ok(a->consts)) return fail(VH_E_ARG, "vh_srnl_sequence_fwd: invalid recurrence constants");
    if ((int64_t)a->length > (int64_t)1 << 30 || (int64_t)a->batch * a->heads > (int64_t)1 << 30)
        return fail(VH_E_RANGE, "vh_srnl_sequence_fwd: sizes exceed the supported range");
    const int vbx = row_vec_bytes(a->head_dim, a->x_dtype), vbq = row_vec_bytes(a->head_dim, a->q_dtype);
    if (!aligned(a->x, vbx) || !aligned(a->y, vbx) || !aligned(a->q, vbq))
        return fail(VH_E_ALIGN, "vh_srnl_sequence_fwd: x/q/y pointers misaligned");

    ScanParams p{};
    p.Mm = a->mem.m; p.Mv = a->mem.v; p.Mk = a->mem.k; p.Me = a->mem.eta; p.Ma = a->mem.alpha;
    p.mem_per_chain = a->mem.per_chain != 0;
    p.x = a->x; p.q = a->q; p.y = a->y;
    p.q_mode = a->q_mode;
    p.B = a->batch; p.R = a->dirs; p.heads = a->heads; p.L = a->length;
    p.C = a->heads * a->head_dim;
    for (int r = 0; r < 4; ++r) p.chunk[r] = r < a->dirs ? a->chunk[r] : 1;
    p.k = to_consts(a->consts);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->q_mode == 1) {
        switch (a->x_dtype) {
            case VH_F32: return sequence_dispatch_d<float, float>(a->head_dim, p, st);
            case VH_BF16: return sequence_dispatch_d<__nv_bfloat16, float>(a->head_dim, p, st);
            default: return sequence_dispatch_d<__half, float>(a->head_dim, p, st);
        }
    }
    switch (a->x_dtype) {
        case VH_F32: return sequence_dispatch_d<float, float>(a->head_dim, p, st);
        case VH_BF16: return sequence_dispatch_d<__nv_bfloat16, __nv_bfloat16>(a->head_dim, p, st);
        default: return sequence_dispatch_d<__half, __half>(a->head_dim, p, st);
    }
}
