"""Channels-last LayerNorm over C with fp32 output (mirror of utils/layer_norm_cuda.py).

The reference's Triton kernels are replaced by ``vh_layernorm_fwd`` (layer_norm_cuda.py:31-57)
and, on the autograd path, ``vh_layernorm_bwd`` (layer_norm_cuda.py:59-119).
"""
import torch

from .. import _lib


@_lib.on_input_device
def layernorm_rows(x_rows, weight, bias, eps, *, want_stats=False, out_dtype=torch.float32):
    """x_rows [rows, C] (any float dtype, contiguous) -> [rows, C] (and mean, rstd).

    out_dtype float32 is the reference's output; bfloat16/float16 round that result once.
    """
    _lib.ensure_device(x_rows)
    x = x_rows.contiguous()
    rows, C = x.shape
    w = weight.detach().reshape(-1).contiguous().float()
    b = bias.detach().reshape(-1).contiguous().float()
    y = torch.empty((rows, C), device=x.device, dtype=out_dtype)
    mean = torch.empty((rows,), device=x.device, dtype=torch.float32) if want_stats else None
    rstd = torch.empty((rows,), device=x.device, dtype=torch.float32) if want_stats else None
    _lib.check(_lib.load().vh_layernorm_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), b.data_ptr(), float(eps), y.data_ptr(),
        _lib.dtype_code(out_dtype), _lib.ptr(mean), _lib.ptr(rstd), rows, C,
        _lib.stream_handle(x.device)), "vh_layernorm_fwd")
    return (y, mean, rstd) if want_stats else y


@_lib.on_input_device
def add_layernorm_rows(x_rows, r_rows, weight, bias, eps, *, out_dtype=torch.float32, sum_out=None):
    """s = x + r (written to ``sum_out``, default x itself) and LayerNorm(s): the block's
    residual add followed by its second norm (models/block.py:105-106).  x, r: contiguous
    [rows, C] fp32/bf16 CUDA tensors, C a multiple of 8.  Returns (s, y)."""
    _lib.ensure_device(x_rows)
    rows, C = x_rows.shape
    if r_rows.shape != x_rows.shape or not x_rows.is_contiguous() or not r_rows.is_contiguous():
        raise RuntimeError("add_layernorm_rows expects two contiguous [rows, C] tensors of one shape")
    s = x_rows if sum_out is None else sum_out
    w = weight.detach().reshape(-1).contiguous().float()
    b = bias.detach().reshape(-1).contiguous().float()
    y = torch.empty((rows, C), device=x_rows.device, dtype=out_dtype)
    _lib.check(_lib.load().vh_add_layernorm_fwd(
        x_rows.data_ptr(), _lib.dtype_code(x_rows.dtype), r_rows.data_ptr(), _lib.dtype_code(r_rows.dtype),
        s.data_ptr(), w.data_ptr(), b.data_ptr(), float(eps), y.data_ptr(), _lib.dtype_code(out_dtype), rows, C,
        _lib.stream_handle(x_rows.device)), "vh_add_layernorm_fwd")
    return s, y


@_lib.on_input_device
def _layernorm2d_forward(x, weight, bias, eps, want_stats=False):
    batch, channels, height, width = x.shape
    rows = x.permute(0, 2, 3, 1).reshape(batch * height * width, channels)
    res = layernorm_rows(rows, weight, bias, eps, want_stats=want_stats)
    y = res[0] if want_stats else res
    y = y.view(batch, height, width, channels).permute(0, 3, 1, 2)
    return (y, res[1], res[2]) if want_stats else y


@_lib.on_input_device
def layernorm_rows_backward(dy_rows, x_rows, weight, mean, rstd):
    """Gradients of :func:`layernorm_rows` (``vh_layernorm_bwd``, replaces the Triton kernels of
    utils/layer_norm_cuda.py:59-119): dy_rows [rows, C] (cast to fp32), the forward's x_rows,
    weight and statistics.  Returns (dx in x's dtype, dweight, dbias fp32 [C])."""
    rows, C = x_rows.shape
    g = dy_rows.contiguous().float()
    x = x_rows.contiguous()
    w = weight.detach().reshape(-1).contiguous().float()
    dx = torch.empty_like(x)
    dw = torch.empty((C,), device=x.device, dtype=torch.float32)
    db = torch.empty((C,), device=x.device, dtype=torch.float32)
    nbytes = int(_lib.load().vh_layernorm_bwd_workspace_bytes(rows, C))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_layernorm_bwd(
        g.data_ptr(), x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
        dx.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(), ws.numel() * 4, rows, C,
        _lib.stream_handle(x.device)), "vh_layernorm_bwd")
    return dx, dw, db


class _LayerNorm2dFunction(torch.autograd.Function):
    """LayerNorm2d with its backward (utils/layer_norm_cuda.py:122-185)."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        y, mean, rstd = _layernorm2d_forward(x, weight, bias, eps, want_stats=True)
        ctx.save_for_backward(x, weight, mean, rstd)
        ctx.param_meta = (weight.shape, weight.dtype, bias.shape, bias.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, mean, rstd = ctx.saved_tensors
        batch, channels, height, width = x.shape
        dy_rows = dy.contiguous(memory_format=torch.channels_last).permute(0, 2, 3, 1).reshape(-1, channels)
        x_rows = x.permute(0, 2, 3, 1).reshape(-1, channels)
        dx, dw, db = layernorm_rows_backward(dy_rows, x_rows, weight, mean, rstd)
        dx = dx.view(batch, height, width, channels).permute(0, 3, 1, 2)
        wshape, wdtype, bshape, bdtype = ctx.param_meta
        return dx, dw.view(wshape).to(wdtype), db.view(bshape).to(bdtype), None


def can_fuse_layernorm2d(x, weight, bias):
    if x.ndim != 4 or not x.is_cuda:
        return False
    if not x.is_contiguous(memory_format=torch.channels_last):
        return False
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return False
    channels = x.shape[1]
    if channels < 1 or weight is None or bias is None:
        return False
    return (weight.device == x.device and bias.device == x.device
            and weight.is_floating_point() and bias.is_floating_point()
            and weight.numel() == channels and bias.numel() == channels)


def visionhope_layernorm2d(x, weight, bias, eps):
    """fp32 LayerNorm over C of a channels-last [B, C, H, W] tensor; returns channels-last."""
    if not x.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError("visionhope_layernorm2d expects channels-last input")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, weight, bias)):
        return _LayerNorm2dFunction.apply(x, weight, bias, float(eps))
    return _layernorm2d_forward(x, weight, bias, float(eps))
