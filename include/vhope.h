/* vhope.h -- C ABI of libvhope.so, the sm_100a implementation of VisionHOPE's inference
 * hot path: the SRNL five-memory recurrence run as four directional chunked scans, spatial
 * restoration and channel-wise direction fusion, query normalization, GRN and LayerNorm.
 *
 * Conventions (every entry point):
 *   - Plain device pointers, element counts and element strides; no framework types.
 *   - The caller allocates every output (the reference allocated inside each op, e.g.
 *     models/srnl_core/csrc/fused.cu:334-335; here ownership moves to the caller so that
 *     calls can be captured in CUDA graphs and hosts without an allocator can use them).
 *   - Work is enqueued on `stream`; nothing synchronizes the host.
 *   - Return 0 on success, a negative VH_E* code when validation rejects the call (nothing
 *     was launched), or a positive cudaError_t when a launch failed.  vh_last_error()
 *     returns a thread-local description of the most recent failure on this thread.
 *   - Call vh_init(device) once per device before capturing any call in a CUDA graph; it
 *     sets the kernels' shared-memory attributes (the reference did this on every call,
 *     fused.cu:23-29).
 *   - Stateless apart from that one-time set-up; thread-safe across streams.
 */
#ifndef VHOPE_H_
#define VHOPE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* vh_stream_t; /* a cudaStream_t */

enum vh_dtype { VH_F32 = 0, VH_BF16 = 1, VH_F16 = 2 };

enum vh_status {
    VH_OK = 0,
    VH_E_ARG = -1,      /* null pointer, bad enum, non-positive size */
    VH_E_SHAPE = -2,    /* inconsistent shapes */
    VH_E_DTYPE = -3,    /* unsupported dtype combination */
    VH_E_HEADDIM = -4,  /* head_dim not in {4, 8, 16, 32, 64} */
    VH_E_ALIGN = -5,    /* pointer or stride misaligned for vector access */
    VH_E_RANGE = -6,    /* sizes beyond the supported index range */
    VH_E_DEVICE = -7    /* device query / attribute set-up failed */
};

/* Recurrence constants (models/srnl_core/chunk.py:44-49, env-overridable there; runtime
 * arguments here).  spectral_factor = 2 * spectral_margin (fused.py:61). */
typedef struct {
    float step_scale;       /* VISIONHOPE_STEP_SCALE, 0.025 */
    float min_retention;    /* VISIONHOPE_MIN_RETENTION, 0.0 */
    float retention_bias;   /* VISIONHOPE_RETENTION_BIAS, 2.197224577 */
    float injection_margin; /* VISIONHOPE_INJECTION_MARGIN, 0.999 */
    float spectral_factor;  /* 2 * VISIONHOPE_SPECTRAL_MARGIN, 1.999998 */
    int32_t spectral_clamp; /* SPECTRAL_CLAMP, 1 */
} vh_srnl_consts;

/* The five initial memories of one SRNL module, fp32, contiguous.
 * Matrices [dirs, heads, D, D] (content m, value v, key k), vectors [dirs, heads, D]
 * (learning rate eta, retention alpha): models/srnl.py:55-68 (core order m, v, k, eta, alpha).
 * per_chain != 0 selects one state per (batch, dir, head) chain, [B, dirs, heads, ...]
 * (models/srnl_core/chunk.py:193-200, StateCount == N). */
typedef struct {
    const float* m;
    const float* v;
    const float* k;
    const float* eta;
    const float* alpha;
    int32_t per_chain;
} vh_srnl_memories;

/* ---------------------------------------------------------------------------------------
 * Fused four-direction spatial operator.
 * Replaces models/srnl_core/csrc/fused.cu:307-351 `srnl_line_forward_seq_noatomic`
 * (kernels parallel_line.cuh:26-59 + merge fused.cu:47-59), bound at
 * models/operator.py:190 through models/srnl_core/fused.py:69-93.
 *
 *   out[b, h, w, c] = sum_d weight[d, c] * (y_d + skip_d[c] * x_d)   at the restored pixel,
 *
 * where y_d is the SRNL output of scan d: 0 row-major, 1 reversed row-major, 2 column-major,
 * 3 reversed column-major (models/operator.py:79-86), chunk = W for rows, H for columns.
 *
 * Input addressing: element (b, d, t, head, i) -- batch b, scan d, token t, head, channel i
 * of the head (unit stride) -- is read at
 *   base + b*batch_stride + d*dir_stride + t*token_stride + head*head_stride + i.
 *   remap == 0: x, q hold the four scans, e.g. [B, 4, L, C] (the reference's
 *               srnl_line_forward_seq* layout: token_stride C, head_stride D) or packed
 *               [B, 4, heads, L, D] (srnl_line_forward*: token_stride D, head_stride L*D).
 *   remap == 1: x, q hold one image in row-major pixel order, e.g. channels-last
 *               [B, H*W, C]; each scan reads it through its own index map (t -> pixel) and
 *               dir_stride is ignored.
 * x and q share dtype (VH_F32 / VH_BF16 / VH_F16).  out: fp32 [B, H, W, C], caller-allocated
 * with out_batch_stride elements per image and C per pixel.
 * skip: C values (shared across directions) or 4*C (skip_per_dir = 1); weight: fp32 [4, C].
 *
 * Optional fields (leave zero / NULL when unused):
 *   aux:       fp32 workspace of three planes with out's layout, plane k at
 *              aux + k * batch * out_batch_stride.  With it (head_dim 16, bf16) the four scans
 *              of a (batch, head) run concurrently in one launch, each into its own plane
 *              (scan 0 into out), and the four planes are summed at the end.  Its content
 *              afterwards is unspecified.  Without it a rows pass and a columns pass run one
 *              after the other, accumulating in out.
 *   final_out: final_dtype [B, H, W, C] with final_batch_stride elements per image and C per
 *              pixel: receives (final_dtype)(sum of the four scans + addend).  out is then
 *              scratch and its content afterwards unspecified.
 *   addend:    io_dtype [B, H, W, C] (addend_batch_stride, C per pixel) added before the
 *              final cast (the block's output position term); requires final_out.
 * -------------------------------------------------------------------------------------*/
typedef struct {
    vh_srnl_memories mem;
    const void* x;
    const void* q;
    int64_t x_batch_stride, x_dir_stride, x_token_stride, x_head_stride;
    int64_t q_batch_stride, q_dir_stride, q_token_stride, q_head_stride;
    int32_t io_dtype;
    int32_t remap;
    const float* skip;
    int32_t skip_per_dir;
    const float* weight;
    float* out;
    int64_t out_batch_stride;
    int32_t batch, height, width, heads, head_dim;
    vh_srnl_consts consts;
    float* aux;
    const void* addend;
    int64_t addend_batch_stride;
    void* final_out;
    int32_t final_dtype;
    int64_t final_batch_stride;
} vh_srnl_spatial_args;

int vh_srnl_spatial_fwd(const vh_srnl_spatial_args* args, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Packed-sequence recurrence (no fusion), y in the dtype of x:
 *   x: [B, R, heads, L, D] packed (models/srnl.py:183-185), R in {1, 2, 4};
 *   q_mode 0: raw queries [B, R, L, C] normalized inside (query_normalization folded in);
 *   q_mode 1: unit-norm fp32 queries [B, R, heads, L, D];
 *   chunk[r]: chunk length of direction r; tokens past L are zero (tail padding).
 * Replaces, forward only:
 *   models/srnl_core/csrc/fused.cu:131-179 `srnl_sequence_forward` (fused.py:96-106),
 *   models/srnl_core/csrc/chunk.cu:1083-1131 `srnl_forward` / `srnl_forward_qraw`
 *     (chunk.py:172-284, 366-505: srnl_normalized_query / srnl_raw_query),
 *   models/srnl_core/csrc/lines.cu:3-237 large/varline forward (lines.py:183-671:
 *     srnl_long_chunk / srnl_variable_lines).
 * -------------------------------------------------------------------------------------*/
typedef struct {
    vh_srnl_memories mem;
    const void* x;
    const void* q;
    void* y;
    int32_t x_dtype;  /* dtype of x and y */
    int32_t q_dtype;  /* == x_dtype for q_mode 0; VH_F32 for q_mode 1 */
    int32_t q_mode;
    int32_t batch, dirs, heads, length, head_dim;
    int32_t chunk[4];
    vh_srnl_consts consts;
} vh_srnl_sequence_args;

int vh_srnl_sequence_fwd(const vh_srnl_sequence_args* args, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Query normalization + relayout, replaces utils/csrc/query_normalization.cu:136-178,
 * 223-265 `visionhope_qnorm_forward` (utils/query_normalization.py:53-90):
 *   q_raw [B, R, L, C] (f32/bf16/f16) -> out fp32 [B, R, heads, L, D] = q / max(||q||, 1e-12),
 *   inv_norm fp32 [B*R*L*heads] (may be NULL).
 * -------------------------------------------------------------------------------------*/
int vh_qnorm_fwd(const void* q_raw, int32_t q_dtype, float* out, float* inv_norm, int32_t batch,
                 int32_t dirs, int32_t length, int32_t heads, int32_t head_dim, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Direction restoration + skip + scale fusion, replaces utils/csrc/direction_fusion.cu:
 * 11-65, 505-575 `visionhope_postprocess_scale_forward` (utils/direction_fusion.py:84-145):
 *   y, x: [B, 4, heads, L, D] (same dtype), skip fp32 C or 4*C values, scale fp32 [4, C];
 *   out fp32 logical [B, C, H, W]: channels_last == 0 -> contiguous NCHW,
 *   channels_last != 0 -> physical [B, H, W, C].
 * -------------------------------------------------------------------------------------*/
int vh_dirfuse_fwd(const void* y, const void* x, int32_t io_dtype, const float* skip,
                   int32_t skip_per_dir, const float* scale, float* out, int32_t channels_last,
                   int32_t batch, int32_t heads, int32_t height, int32_t width, int32_t head_dim,
                   vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Global response norm on channels-last input, fp32 output; replaces utils/csrc/
 * grn_cuda.cu:46-124, 267-300 `grn_forward_cuda` (utils/grn_cuda.py:103-117, utils/grn.py:41-70):
 *   x physical [B, H, W, C] (f32/bf16/f16), gamma/beta fp32 [C], y fp32 [B, H, W, C];
 *   y = x * (1 + gamma * Gx / (mean_c Gx + eps)) + beta, Gx[b,c] = ||x[b,:,:,c]||_2.
 *   y_dtype: VH_F32 (the reference's output) or VH_BF16/VH_F16, the same fp32 result rounded
 *   once -- what an autocast consumer would cast it to.
 *   gx (fp32 [B, C]) and inv_den (fp32 [B]) receive the statistics (the reference saves them
 *   for backward); both may be NULL.
 *   workspace: caller-provided device scratch of vh_grn_workspace_bytes(...) bytes.
 * -------------------------------------------------------------------------------------*/
int64_t vh_grn_workspace_bytes(int32_t batch, int32_t height, int32_t width, int32_t channels);
int vh_grn_fwd(const void* x, int32_t x_dtype, const float* gamma, const float* beta, float eps,
               void* y, int32_t y_dtype, float* gx, float* inv_den, void* workspace, int64_t workspace_bytes,
               int32_t batch, int32_t height, int32_t width, int32_t channels, vh_stream_t stream);

/* GRN from precomputed statistics: the apply pass of vh_grn_fwd when the sums of x^2 per
 * (image, channel) were produced with x itself (vh_dwconv_fwd's `sumsq`).  sumsq: fp32
 * [B, nparts, C], sums over disjoint pixel slices of each image, added in slice order;
 * Gx = sqrt(sum), f = 1 + gamma Gx / (mean_c Gx + eps) is written to `factors` (fp32 [B, C],
 * 16-byte aligned) and y = x f + beta  (grn_cuda.cu:46-124).  x, y: dense channels-last
 * [B, H, W, C], 16-byte aligned, y distinct from x; C a multiple of 8, at most 2048. */
int vh_grn_apply_fwd(const void* x, int32_t x_dtype, const float* sumsq, int32_t nparts,
                     const float* gamma, const float* beta, float eps, float* factors, void* y,
                     int32_t y_dtype, int32_t batch, int32_t height, int32_t width, int32_t channels,
                     vh_stream_t stream);

/* GRN that allocates nothing (no counterpart in the reference).  Same result as vh_grn_fwd,
 * for callers that cannot allocate device memory when they run -- plugin or serving hosts
 * whose op interface provides only input and output buffers, and deployments that fix their
 * device memory at start-up.  The partial sums live in a 4 MiB array built into the library
 * (held on every device that loads it until the process exits), so batch * channels must not
 * exceed 1,048,576; larger calls are rejected with VH_E_RANGE.  The first call on each device
 * looks up that array's device address once (make that first call before any stream capture).
 * All calls share the one array: calls that may overlap on the GPU (different streams, or
 * different host threads on one device) race and must be serialized by the caller; the array
 * keeps the last call's contents, which no call relies on.  The looked-up address is kept for
 * the life of the process: after cudaDeviceReset, or after the device's primary context is
 * destroyed and created again, the array may sit at another address, so such a caller must
 * call vh_grn_noalloc_reset() (on any thread) before its next call. */
int vh_grn_fwd_noalloc(const void* x, int32_t x_dtype, const float* gamma, const float* beta,
                       float eps, float* y, float* gx, float* inv_den, int32_t batch,
                       int32_t height, int32_t width, int32_t channels, vh_stream_t stream);
/* Forget the device addresses vh_grn_fwd_noalloc looked up (see above); the next call on
 * each device looks its array up again.  No counterpart in the reference. */
void vh_grn_noalloc_reset(void);

/* ---------------------------------------------------------------------------------------
 * LayerNorm over the channel axis of channels-last rows, fp32 output; replaces the Triton
 * kernel utils/layer_norm_cuda.py:31-57, 122-147 `visionhope_layernorm2d` and the
 * F.layer_norm path of models/layers.py:17-35:
 *   x [rows, C] (f32/bf16/f16), weight/bias fp32 [C], y [rows, C] of y_dtype (VH_F32 is the
 *   reference's output; VH_BF16/VH_F16 round the fp32 result once); mean/rstd fp32 [rows]
 *   (may be NULL).
 * -------------------------------------------------------------------------------------*/
int vh_layernorm_fwd(const void* x, int32_t x_dtype, const float* weight, const float* bias,
                     float eps, void* y, int32_t y_dtype, float* mean, float* rstd, int64_t rows,
                     int32_t channels, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Depthwise KxK convolution (stride 1, zero padding K/2, one filter per channel) of a
 * channels-last image with the elementwise work that follows it in the VisionHOPE block
 * fused into the same pass; replaces the nn.Conv2d(groups=C) calls of models/block.py
 * (cpe :100, local_conv :57-62, local_position :78) and of the FFN's depthwise stage
 * (models/layers.py, FeedForward), together with their bias, activation, gate and residual
 * operations:
 *   VH_DW_BIAS   y = conv(x) + b
 *   VH_DW_RESID  y = x + (conv(x) + b)
 *   VH_DW_GATE   y = x + sigmoid(gate) * (conv(x) + b)
 *   VH_DW_GELU   h = gelu(x);  y = gelu(h + conv(h) + b)      (gelu: exact erf form)
 *   VH_DW_RESID_ADD  s = x + r (r in `gate`, gate_dtype);  y = s + (conv(s) + b): the block's
 *                cpe applied to the previous block's output without materialising it
 *   VH_DW_GATE_POS  y as VH_DW_GATE, then pos_y = conv_pos(y) + pos_bias from the same CTA's
 *                copy of y (the block's local features followed by its output position
 *                term, models/block.py:57-62 and :78).  bf16 only, ksize 7, pos_ksize 5, and
 *                whole images per CTA: H = W = 14 or H = W = 7.  Bit-identical to VH_DW_GATE
 *                followed by VH_DW_BIAS on y.
 * x, gate, y: dense [B, H, W, C] of `dtype` (VH_F32 or VH_BF16), 16-byte aligned, y distinct
 * from the inputs; weight fp32 [C, K, K] (nn.Conv2d's [C, 1, K, K]); bias fp32 [C];
 * C a multiple of 8.  The convolution reads input, weight and bias rounded to bf16 and sums in
 * fp32 (a bf16 convolution under autocast); the residual and gate terms use x and gate as
 * given; y is rounded once.
 * -------------------------------------------------------------------------------------*/
enum vh_dw_mode { VH_DW_BIAS = 0, VH_DW_RESID = 1, VH_DW_GATE = 2, VH_DW_GELU = 3, VH_DW_RESID_ADD = 4,
                  VH_DW_GATE_POS = 5 };

typedef struct {
    const void* x;
    const void* gate;
    const float* weight;
    const float* bias;
    void* y;
    int32_t dtype;
    int32_t mode;
    int32_t ksize;
    int32_t batch, height, width, channels;
    int32_t gate_dtype; /* VH_DW_RESID_ADD: dtype of the addend r (fp32 or bf16) */
    /* VH_DW_GELU only, may be NULL: fp32 [B, vh_dwconv_tiles(H, W), C] receiving, per image and
     * pixel tile, the sum over the tile of y^2 per channel, with y as stored (the statistics
     * pass of a GRN that follows, see vh_grn_apply_fwd).  Written, not accumulated. */
    float* sumsq;
    /* VH_DW_GATE_POS only (NULL / 0 otherwise): the second depthwise convolution's weight fp32
     * [C, pos_ksize, pos_ksize], bias fp32 [C] and output [B, H, W, C] of `dtype`. */
    const float* pos_weight;
    const float* pos_bias;
    void* pos_y;
    int32_t pos_ksize;
} vh_dwconv_args;

int vh_dwconv_fwd(const vh_dwconv_args* args, vh_stream_t stream);

/* Number of pixel tiles per image that vh_dwconv_fwd uses for an H x W image (the middle
 * extent of its `sumsq` output). */
int vh_dwconv_tiles(int32_t height, int32_t width);

/* ---------------------------------------------------------------------------------------
 * Bias and activation over channels-last rows: y[r, c] = act(x[r, c] + bias[c]), computed in
 * fp32 and rounded once to y's dtype.  The epilogue of a convolution with its eval-mode
 * BatchNorm folded in (the stem and downsample layers of models/layers.py:85-107: conv, BN,
 * GELU).  act: VH_ACT_NONE or VH_ACT_GELU (exact erf form).  x, y: [rows, C], C a multiple of
 * 8, 16-byte aligned; bias fp32 [C].
 * -------------------------------------------------------------------------------------*/
enum vh_act { VH_ACT_NONE = 0, VH_ACT_GELU = 1 };

int vh_bias_act_fwd(const void* x, int32_t x_dtype, const float* bias, void* y, int32_t y_dtype,
                    int64_t rows, int32_t channels, int32_t act, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Row GEMM of the block's 1x1 projections: y[M, N] = x[M, K] W[N, K]^T + bias, bf16 x, W and
 * y, fp32 bias (may be NULL), fp32 accumulation and one rounding (F.linear under bf16
 * autocast; models/block.py proj_in / local_gate / proj_out, models/operator.py W_q, the
 * FFN's fc1 / fc2 as 1x1 convolutions of channels-last tensors).  K and N in
 * {32, 64, 128, 256} with K * N <= 32768; x, W, y 16-byte aligned, dense rows.
 * -------------------------------------------------------------------------------------*/
int vh_rows_gemm_fwd(const void* x, const void* weight, const float* bias, void* y, int64_t rows,
                     int32_t in_features, int32_t out_features, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * The block's first LayerNorm and input projection in one pass (models/block.py:104, norm1
 * then proj_in; norm: models/layers.py:9-35, projection: the 1x1 convolution proj_in):
 *   y[M, N] = bf16(LayerNorm(x)[M, K]) W[N, K]^T + bias,
 * LayerNorm over each row's K channels (biased variance, eps inside the square root, fp32
 * ln_weight / ln_bias), its result rounded to bf16 as the projection under bf16 autocast reads
 * it, then the row GEMM's arithmetic (fp32 accumulation, fp32 bias may be NULL, one rounding).
 * x: fp32 [M, K] (the residual stream); W, y bf16.  K in {32, 64, 128}, N in {32, 64}; x, W,
 * y, ln_weight and ln_bias 16-byte aligned, dense rows.  The normalized rows are not written.
 * -------------------------------------------------------------------------------------*/
int vh_ln_rows_gemm_fwd(const float* x, const float* ln_weight, const float* ln_bias, float eps,
                        const void* weight, const float* bias, void* y, int64_t rows,
                        int32_t in_features, int32_t out_features, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * First stem layer with its BatchNorm folded in (models/layers.py:85-107): a 3x3 convolution,
 * stride 2, padding 1, of a 3-channel image, then bias and activation:
 *   y = act(bf16(conv(bf16(x), bf16(w))) + bias), rounded once to y_dtype
 * (the arithmetic of the convolution under bf16 autocast followed by vh_bias_act_fwd).
 * x: fp32 [B, H, W, 3] (channels-last image); weight fp32 [C_out, 3, 3, 3] (nn.Conv2d's);
 * bias fp32 [C_out]; y: [B, (H+1)/2, (W+1)/2, C_out] of y_dtype (VH_F32 or VH_BF16);
 * C_out in {16, 24, 32, 48, 64}; act VH_ACT_NONE or VH_ACT_GELU.
 * -------------------------------------------------------------------------------------*/
int vh_stem_conv_fwd(const float* x, const float* weight, const float* bias, void* y, int32_t y_dtype,
                     int32_t batch, int32_t height, int32_t width, int32_t out_channels, int32_t act,
                     vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Residual add with a cast: y = (y_dtype)(x + r), summed in fp32 and rounded once
 * (models/block.py:106, the last block's `x + branch` of a stage, fused with the autocast cast
 * of the downsample convolution that reads it).  x, r, y: n elements each (n a multiple of 8),
 * fp32 or bf16, 16-byte aligned; y distinct from x and r.
 * -------------------------------------------------------------------------------------*/
int vh_add_cast_fwd(const void* x, int32_t x_dtype, const void* r, int32_t r_dtype, void* y, int32_t y_dtype,
                    int64_t n, vh_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Residual add followed by LayerNorm over channels-last rows (models/block.py:105-106, the
 * block's `x + branch` then `norm2`):  s = x + r is written to sum_out (x's dtype; may be x
 * itself) and y = LayerNorm(s) to y (y_dtype), with the statistics of the stored s.
 * x, sum_out: [rows, C] of x_dtype; r: [rows, C] of r_dtype; C a multiple of 8; all
 * 16-byte aligned.
 * -------------------------------------------------------------------------------------*/
int vh_add_layernorm_fwd(const void* x, int32_t x_dtype, const void* r, int32_t r_dtype, void* sum_out,
                         const float* weight, const float* bias, float eps, void* y, int32_t y_dtype,
                         int64_t rows, int32_t channels, vh_stream_t stream);

/* =======================================================================================
 * Backward (training) entry points.  Every reduction runs in a fixed order, so gradients are
 * bit-reproducible; the ones that reduce over pixels or rows take a caller-provided workspace
 * of the size their *_workspace_bytes function gives.
 * =====================================================================================*/

/* SRNL recurrence backward for packed sequences (head_dim 16: any chunk length; head_dim 4, 8
 * or 32: chunks of up to 64 tokens); replaces models/srnl_core/csrc/chunk.cu:511-1057,
 * 1133-1206 `srnl_backward` / `srnl_backward_qraw` (chunk.py:286-359
 * SRNLNormalizedQueryFunction.backward, 507-588 SRNLRawQueryFunction.backward) and
 * models/srnl_core/csrc/lines.cu:252-669 (lines.py: srnl_long_chunk, srnl_variable_lines).  The
 * inputs are the forward's (mem, x, q, q_mode, sizes, chunks, consts: see
 * vh_srnl_sequence_args); nothing from the forward is saved besides them: the chunk states and
 * the gain sequence are recomputed.  For head_dim 16 the workspace holds the whole gain history
 * when that fits 6 GiB (environment variable VHOPE_SRNL_BWD_HISTORY_BYTES sets the budget; 0
 * keeps one chunk's history and recomputes it per chunk); the workspace size and the call must
 * see the same setting.  grad_y fp32 [B, R, heads, L, D].
 * Writes grad_x (fp32, x's shape), grad_q (fp32, q's shape: [B, R, L, C] for raw queries,
 * through their normalization; [B, R, heads, L, D] for normalized ones) and grad_m, grad_v,
 * grad_k, grad_eta, grad_alpha (fp32, the memories' shapes; shared memories get the sum over the
 * batch).  workspace: vh_srnl_sequence_bwd_workspace_bytes(args) bytes. */
typedef struct {
    vh_srnl_memories mem;
    const void* x;
    const void* q;
    int32_t x_dtype;
    int32_t q_dtype;
    int32_t q_mode;
    const float* grad_y;
    float* grad_x;
    float* grad_q;
    float* grad_m;
    float* grad_v;
    float* grad_k;
    float* grad_eta;
    float* grad_alpha;
    int32_t batch, dirs, heads, length, head_dim;
    int32_t chunk[4];
    vh_srnl_consts consts;
} vh_srnl_sequence_bwd_args;

int64_t vh_srnl_sequence_bwd_workspace_bytes(const vh_srnl_sequence_bwd_args* args);
int vh_srnl_sequence_bwd(const vh_srnl_sequence_bwd_args* args, void* workspace, int64_t workspace_bytes,
                         vh_stream_t stream);

/* Query normalization backward; replaces utils/csrc/query_normalization.cu:78-134, 180-221,
 * 267-300 `visionhope_qnorm_backward` (utils/query_normalization.py:68-76):
 *   grad_out, q_out fp32 [B, R, heads, L, D]; inv_norm fp32 [B*R*L*heads] (vh_qnorm_fwd's);
 *   grad_q [B, R, L, C] of q_dtype = (g - q_out (q_out . g)) inv (g inv where the norm was
 *   clamped, inv = 1e12). */
int vh_qnorm_bwd(const float* grad_out, const float* q_out, const float* inv_norm, void* grad_q, int32_t q_dtype,
                 int32_t batch, int32_t dirs, int32_t length, int32_t heads, int32_t head_dim, vh_stream_t stream);

/* Direction restoration + fusion backward; replaces utils/csrc/direction_fusion.cu:123-502,
 * 577-691 `visionhope_postprocess_scale_backward` (utils/direction_fusion.py:106-118):
 *   grad_out fp32 logical [B, C, H, W] with element strides gs_b, gs_c, gs_h, gs_w (any layout);
 *   y, x [B, 4, heads, L, D] of io_dtype; skip (C or 4*C values, skip_per_dir) and scale [4, C]
 *   fp32.  Writes grad_y, grad_x (io_dtype, y's layout) and grad_skip, grad_scale (fp32, the
 *   shapes of skip and scale).  workspace: vh_dirfuse_bwd_workspace_bytes(...) bytes. */
int64_t vh_dirfuse_bwd_workspace_bytes(int32_t batch, int32_t heads, int32_t height, int32_t width,
                                       int32_t head_dim);
int vh_dirfuse_bwd(const float* grad_out, int64_t gs_b, int64_t gs_c, int64_t gs_h, int64_t gs_w, const void* y,
                   const void* x, int32_t io_dtype, const float* skip, int32_t skip_per_dir, const float* scale,
                   void* grad_y, void* grad_x, float* grad_skip, float* grad_scale, void* workspace,
                   int64_t workspace_bytes, int32_t batch, int32_t heads, int32_t height, int32_t width,
                   int32_t head_dim, vh_stream_t stream);

/* LayerNorm over channels-last rows, backward; replaces the Triton kernels
 * utils/layer_norm_cuda.py:59-119, 150-185 (`_layernorm2d_backward_kernel`,
 * `_layernorm2d_reduce_kernel`):  grad_y fp32 [rows, C]; x [rows, C] of x_dtype; weight fp32
 * [C]; mean, rstd fp32 [rows] (vh_layernorm_fwd's).  Writes grad_x (x_dtype) and grad_weight,
 * grad_bias (fp32 [C]).  workspace: vh_layernorm_bwd_workspace_bytes(rows, C) bytes. */
int64_t vh_layernorm_bwd_workspace_bytes(int64_t rows, int32_t channels);
int vh_layernorm_bwd(const float* grad_y, const void* x, int32_t x_dtype, const float* weight, const float* mean,
                     const float* rstd, void* grad_x, float* grad_weight, float* grad_bias, void* workspace,
                     int64_t workspace_bytes, int64_t rows, int32_t channels, vh_stream_t stream);

/* GRN backward; replaces utils/csrc/grn_cuda.cu:126-265, 322-359 `grn_backward_cuda`
 * (utils/grn_cuda.py:49-80):  grad_y fp32 and x (x_dtype) channels-last [B, H, W, C]; gamma
 * fp32 [C]; gx fp32 [B, C] and inv_den fp32 [B] (vh_grn_fwd's statistics).  Writes grad_x
 * (x_dtype), grad_gamma and grad_beta (fp32 [C]).  workspace: vh_grn_bwd_workspace_bytes(B, C)
 * bytes. */
int64_t vh_grn_bwd_workspace_bytes(int32_t batch, int32_t channels);
int vh_grn_bwd(const float* grad_y, const void* x, int32_t x_dtype, const float* gamma, const float* gx,
               const float* inv_den, void* grad_x, float* grad_gamma, float* grad_beta, void* workspace,
               int64_t workspace_bytes, int32_t batch, int32_t height, int32_t width, int32_t channels,
               vh_stream_t stream);

/* LayerScale residual add; replaces the Triton kernel utils/residual.py:30-52
 * (`_residual_forward_kernel`, launched at residual.py:107-129):  residual (residual_dtype) and
 * branch (branch_dtype) channels-last [B, S, C]; gamma fp32 [C]; drop_scale fp32 [B] (the
 * drop-path keep mask, already divided by the keep probability).  Writes out fp32 [B, S, C] =
 * residual + branch * gamma * drop_scale. */
int vh_residual_add_fwd(const void* residual, int32_t residual_dtype, const void* branch, int32_t branch_dtype,
                        const float* gamma, const float* drop_scale, float* out, int32_t batch, int64_t spatial,
                        int32_t channels, vh_stream_t stream);

/* LayerScale residual add, backward; replaces utils/residual.py:54-101, 131-169
 * (`_residual_backward_kernel`, `_residual_reduce_kernel`):  grad_out fp32 [B, S, C]; branch
 * (branch_dtype), gamma, drop_scale as in the forward.  Writes grad_branch (branch_dtype) =
 * grad_out * gamma * drop_scale and grad_gamma fp32 [C]; the residual's gradient is grad_out
 * itself.  workspace: vh_residual_add_bwd_workspace_bytes(B * S, C) bytes. */
int64_t vh_residual_add_bwd_workspace_bytes(int64_t rows, int32_t channels);
int vh_residual_add_bwd(const float* grad_out, const void* branch, int32_t branch_dtype, const float* gamma,
                        const float* drop_scale, void* grad_branch, float* grad_gamma, void* workspace,
                        int64_t workspace_bytes, int32_t batch, int64_t spatial, int32_t channels,
                        vh_stream_t stream);

/* Measurement helper (no reference counterpart): launches `blocks` x 256 threads, each
 * running 32 * iters dependent-free FMAs; out needs blocks * 256 floats.  bench.py times it
 * to measure the device's FP32 (non-tensor) FMA peak. */
int vh_probe_ffma(float* out, int32_t blocks, int32_t iters, vh_stream_t stream);

/* One-time per-device set-up (kernel shared-memory attributes).  Idempotent. */
int vh_init(int32_t device);

/* Thread-local description of the last failure on this thread ("" if none). */
const char* vh_last_error(void);

/* Number of kernels the last entry point called on this thread launched (0 after a
 * validation failure).  Lets a host count device launches without knowing each path. */
int vh_last_launch_count(void);

/* Status of the chunk-parallel tensor-core scan (no counterpart in the reference): non-zero
 * once, on any launch since the last reset, one of its bounded waits (a TMA tile or tensor-core
 * result that did not arrive within 2 s) gave up; the CTA then stopped its chain, released its
 * tensor memory and left, and that call's output is invalid.  Synchronous (reads a device
 * word); reset != 0 clears it.  Returns -1 when the word cannot be read. */
int vh_tc_status(int32_t reset);

/* Library version string. */
const char* vh_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VHOPE_H_ */
