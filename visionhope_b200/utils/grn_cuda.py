"""GRN on channels-last CUDA tensors with fp32 output (mirror of utils/grn_cuda.py).

``visionhope_grn`` calls ``vh_grn_fwd`` (replaces utils/csrc/grn_cuda.cu:267-300).  The
statistics workspace comes from PyTorch's caching allocator.  The autograd path saves the
forward's statistics and runs ``vh_grn_bwd`` (replaces utils/csrc/grn_cuda.cu:126-265).
"""
import torch

from .. import _lib


@_lib.on_input_device
def grn_forward(x, gamma, beta, eps, *, want_stats=False, out_dtype=torch.float32):
    """x logical [B, C, H, W] stored channels-last -> channels-last y (and Gx, 1/den).

    out_dtype float32 is the reference's output; bfloat16/float16 return the same fp32 result
    rounded once, which is exactly what an autocast consumer would cast it to.
    """
    _lib.ensure_device(x)
    if x.dim() != 4 or not x.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError("GRN CUDA expects channels-last NCHW input")
    B, C, H, W = x.shape
    g = gamma.detach().reshape(-1).contiguous().float()
    b = beta.detach().reshape(-1).contiguous().float()
    if g.numel() != C or b.numel() != C:
        raise RuntimeError("GRN CUDA requires contiguous FP32 channel parameters on the input device")
    y = torch.empty_like(x, dtype=out_dtype, memory_format=torch.channels_last)
    gx = torch.empty((B, C), device=x.device, dtype=torch.float32) if want_stats else None
    inv = torch.empty((B,), device=x.device, dtype=torch.float32) if want_stats else None
    nbytes = int(_lib.load().vh_grn_workspace_bytes(B, H, W, C))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_grn_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), g.data_ptr(), b.data_ptr(), float(eps), y.data_ptr(),
        _lib.dtype_code(out_dtype), _lib.ptr(gx), _lib.ptr(inv), ws.data_ptr(), ws.numel() * 4, B, H, W, C,
        _lib.stream_handle(x.device)), "vh_grn_fwd")
    return (y, gx, inv) if want_stats else y


def grn_apply(x, sumsq, gamma, beta, eps, *, out_dtype=torch.float32):
    """GRN of channels-last ``x`` from its precomputed statistics: ``sumsq`` fp32 [B, P, C]
    holds sums of x^2 per channel over P disjoint pixel slices of each image (as the fused
    depthwise GELU kernel returns them), so x is read once here (``vh_grn_apply_fwd``).
    Same result as :func:`grn_forward` up to the order of the fp32 sums."""
    _lib.ensure_device(x)
    if x.dim() != 4 or not x.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError("GRN CUDA expects channels-last NCHW input")
    B, C, H, W = x.shape
    if sumsq.dtype != torch.float32 or sumsq.dim() != 3 or sumsq.shape[0] != B or sumsq.shape[2] != C:
        raise RuntimeError("grn_apply: sumsq must be fp32 [B, slices, C]")
    sumsq = sumsq.contiguous()
    g = gamma.detach().reshape(-1).contiguous().float()
    b = beta.detach().reshape(-1).contiguous().float()
    y = torch.empty_like(x, dtype=out_dtype, memory_format=torch.channels_last)
    factors = torch.empty((B, C), device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_grn_apply_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), sumsq.data_ptr(), sumsq.shape[1], g.data_ptr(), b.data_ptr(),
        float(eps), factors.data_ptr(), y.data_ptr(), _lib.dtype_code(out_dtype), B, H, W, C,
        _lib.stream_handle(x.device)), "vh_grn_apply_fwd")
    return y


def grn_apply_ok(x):
    """Shapes the statistics-fed GRN takes: channels a multiple of 8, at most 2048."""
    C = x.shape[1]
    return C % 8 == 0 and C <= 2048


@_lib.on_input_device
def grn_backward(dout, x, gamma, gx, inv_den):
    """Gradients of :func:`grn_forward` (``vh_grn_bwd``, replaces utils/csrc/grn_cuda.cu:126-265):
    dout [B, C, H, W] (any float dtype and layout), the forward's x, gamma and its statistics
    Gx [B, C], 1/den [B].  Returns (dx channels-last in x's dtype, dgamma, dbeta fp32 [C])."""
    B, C, H, W = x.shape
    g = dout.to(dtype=torch.float32, memory_format=torch.channels_last)
    dx = torch.empty_like(x, memory_format=torch.channels_last)
    dgamma = torch.empty((C,), device=x.device, dtype=torch.float32)
    dbeta = torch.empty((C,), device=x.device, dtype=torch.float32)
    nbytes = int(_lib.load().vh_grn_bwd_workspace_bytes(B, C))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_grn_bwd(
        g.data_ptr(), x.data_ptr(), _lib.dtype_code(x.dtype), gamma.data_ptr(), gx.data_ptr(), inv_den.data_ptr(),
        dx.data_ptr(), dgamma.data_ptr(), dbeta.data_ptr(), ws.data_ptr(), ws.numel() * 4, B, H, W, C,
        _lib.stream_handle(x.device)), "vh_grn_bwd")
    return dx, dgamma, dbeta


class _GRNFunction(torch.autograd.Function):
    """GRN with its backward (utils/grn_cuda.py:33-80): saves x, gamma and the statistics."""

    @staticmethod
    def forward(ctx, x, gamma, beta, eps):
        y, gx, inv = grn_forward(x, gamma, beta, eps, want_stats=True)
        g = gamma.detach().reshape(-1).contiguous().float()
        ctx.save_for_backward(x, g, gx, inv)
        ctx.param_shapes = (gamma.shape, gamma.dtype, beta.shape, beta.dtype)
        return y

    @staticmethod
    def backward(ctx, dout):
        x, g, gx, inv = ctx.saved_tensors
        dx, dgamma, dbeta = grn_backward(dout, x, g, gx, inv)
        gshape, gdtype, bshape, bdtype = ctx.param_shapes
        return dx, dgamma.view(gshape).to(gdtype), dbeta.view(bshape).to(bdtype), None


def can_fuse_grn(x, gamma, beta):
    if x.ndim != 4 or not x.is_cuda or not x.is_contiguous(memory_format=torch.channels_last):
        return False
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return False
    channels = x.shape[1]
    spatial = x.shape[2] * x.shape[3]
    if x.shape[0] < 1 or x.shape[0] > 65535 or channels < 1 or spatial < 1 or channels % 4:
        return False
    return (gamma.device == x.device and beta.device == x.device
            and gamma.dtype == torch.float32 and beta.dtype == torch.float32
            and gamma.numel() == channels and beta.numel() == channels)


def visionhope_grn(x, gamma, beta, eps):
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, gamma, beta)):
        return _GRNFunction.apply(x, gamma, beta, eps)
    return grn_forward(x, gamma, beta, eps)
