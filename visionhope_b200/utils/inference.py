"""Inference-time helpers of the block harness: GEMMs over channels-last activations with
weights already in the autocast dtype.

Under bf16 autocast every Linear / 1x1-convolution call casts its fp32 weight and bias to
bf16 first (one small kernel per call).  ``cache_half_weights`` makes those bf16 copies once,
when a model is prepared for inference, and ``linear_cached`` uses them whenever autocast would
have made the same cast, so the results are bit-identical to the uncached call.
Re-run the preparation after changing weights.
"""
import torch
from torch.nn import functional as F


def _autocast_bf16():
    return torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16


def _weight_2d(module):
    w = module.weight
    return w if w.dim() == 2 else w[:, :, 0, 0]


def cache_half_weights(module):
    """Keep bf16 copies of a Linear / 1x1 Conv2d weight and bias on the module (and the bf16
    bias widened back to fp32, exactly, for the row GEMM's epilogue)."""
    with torch.no_grad():
        w = _weight_2d(module).detach().to(torch.bfloat16).contiguous()
        b = None if module.bias is None else module.bias.detach().to(torch.bfloat16).contiguous()
    module._vh_half = (w, b)
    module._vh_bias32 = None if b is None else b.float()


_ROW_GEMM_DIMS = (32, 64, 128, 256)
# (in, out) features where the row GEMM measured faster than the library GEMM on B200 at
# VisionHOPE-T's row counts (batch 256): 802816 x 64 -> 32: 31.7 us against 48.1 us;
# 802816 x 32 -> 32: 23.5 against 46.1; 200704 x 64 -> 64: 20.5 against 22.5.  Wider
# projections, and the 50176-row stage-3 ones, stay with cuBLAS.
_ROWS_GEMM_FASTER = {(32, 32), (64, 32), (64, 64)}


def rows_gemm_ok(k, n):
    """Projection shapes the row GEMM kernel takes (``vh_rows_gemm_fwd``)."""
    return k in _ROW_GEMM_DIMS and n in _ROW_GEMM_DIMS and k * n <= 32768


def rows_gemm(x, w, bias32=None):
    """y = x W^T + b over the rows of bf16 ``x`` [..., K] with bf16 ``w`` [N, K] and an fp32
    (widened bf16) bias, fp32 accumulation and one rounding (``vh_rows_gemm_fwd``)."""
    from .. import _lib

    _lib.ensure_device(x)
    n, k = w.shape
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.shape[-1] != k or not rows_gemm_ok(k, n):
        raise RuntimeError("rows_gemm expects bf16 x [..., K], bf16 W [N, K] with K, N in {32..256}, K*N <= 32768")
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    y = torch.empty(x.shape[:-1] + (n,), device=x.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().vh_rows_gemm_fwd(x2.data_ptr(), w.data_ptr(), _lib.ptr(bias32), y.data_ptr(),
                                            x2.shape[0], k, n, _lib.stream_handle(x.device)), "vh_rows_gemm_fwd")
    return y


def ln_rows_gemm_ok(k, n):
    """Shapes the LayerNorm + row GEMM kernel takes (``vh_ln_rows_gemm_fwd``)."""
    return k in (32, 64, 128) and n in (32, 64)


def ln_rows_gemm(x, ln_weight, ln_bias, eps, w, bias32=None):
    """bf16(LayerNorm(x)) W^T + b over the rows of fp32 ``x`` [..., K] in one pass: the
    block's norm1 followed by proj_in under bf16 autocast, without writing the normalized rows
    (``vh_ln_rows_gemm_fwd``).  ``w``: bf16 [N, K]; ``bias32``: the fp32 (widened bf16) bias."""
    from .. import _lib

    _lib.ensure_device(x)
    n, k = w.shape
    if (x.dtype != torch.float32 or w.dtype != torch.bfloat16 or x.shape[-1] != k or not ln_rows_gemm_ok(k, n)
            or ln_weight.numel() != k or ln_bias.numel() != k):
        raise RuntimeError("ln_rows_gemm expects fp32 x [..., K], bf16 W [N, K], K in {32, 64, 128}, N in {32, 64}")
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    lw = ln_weight.detach().reshape(-1).float().contiguous()
    lb = ln_bias.detach().reshape(-1).float().contiguous()
    y = torch.empty(x.shape[:-1] + (n,), device=x.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().vh_ln_rows_gemm_fwd(x2.data_ptr(), lw.data_ptr(), lb.data_ptr(), float(eps), w.data_ptr(),
                                               _lib.ptr(bias32), y.data_ptr(), x2.shape[0], k, n,
                                               _lib.stream_handle(x.device)), "vh_ln_rows_gemm_fwd")
    return y


def norm_linear_cached(norm, module, x):
    """``linear_cached(module, norm(x))`` in one kernel when ``norm`` is a LayerNorm over the
    last dim of fp32 rows ``x`` and the projection's cached bf16 weight has a shape the fused
    kernel takes (under bf16 autocast, autograd off); None otherwise, for the caller to run the
    two operations."""
    cached = getattr(module, "_vh_half", None)
    if (cached is None or x.dtype != torch.float32 or not x.is_cuda or torch.is_grad_enabled()
            or not _autocast_bf16() or cached[0].device != x.device or not x.is_contiguous()):
        return None
    n, k = cached[0].shape
    if not ln_rows_gemm_ok(k, n) or x.shape[-1] != k or norm.weight is None or norm.bias is None:
        return None
    return ln_rows_gemm(x, norm.weight, norm.bias, norm.eps, cached[0], getattr(module, "_vh_bias32", None))


def linear_cached(module, x):
    """``F.linear(x, W, b)`` for a Linear or a 1x1 Conv2d applied to channels-last rows ``x``
    (last dim = in_features), using the cached bf16 weights when x is bf16 under bf16 autocast
    with autograd off."""
    cached = getattr(module, "_vh_half", None)
    if (cached is not None and x.dtype == torch.bfloat16 and x.is_cuda and not torch.is_grad_enabled()
            and _autocast_bf16() and cached[0].device == x.device):
        n, k = cached[0].shape
        if (k, n) in _ROWS_GEMM_FASTER and x.is_contiguous():
            return rows_gemm(x, cached[0], getattr(module, "_vh_bias32", None))
        return F.linear(x, cached[0], cached[1])
    return F.linear(x, _weight_2d(module), module.bias)
