"""Restore and fuse directional SRNL outputs (mirror of utils/direction_fusion.py).

    out = sum_d scale[d] * (y[d] + d_skip[d] * x[d])

computed by ``vh_dirfuse_fwd`` (replaces utils/csrc/direction_fusion.cu:11-65); fp32 output,
logical NCHW, channels-last storage when requested.  The autograd path runs ``vh_dirfuse_bwd``
(direction_fusion.cu:123-502).
"""
import torch

from .. import _lib


@_lib.on_input_device
def _postprocess_forward(y, x, d_skip, direction_scale, height, width, channels_last):
    _lib.ensure_device(y)
    if y.dtype != x.dtype:
        raise RuntimeError("visionhope_postprocess_scale_forward expects matching Y and X dtypes.")
    y_c, x_c = y.contiguous(), x.contiguous()
    skip = d_skip.detach().contiguous().float()
    scale = direction_scale.detach().contiguous().float()
    B, R, heads, L, D = y_c.shape
    C = heads * D
    if skip.numel() not in (C, 4 * C):
        raise RuntimeError("d_skip must contain C or 4*C values")
    if R != 4 or tuple(x_c.shape) != tuple(y_c.shape) or height * width != L or tuple(scale.shape) != (4, C):
        raise RuntimeError("Invalid shape for visionhope_postprocess_scale_forward.")
    if channels_last:
        out = torch.empty_strided((B, C, height, width), (height * width * C, 1, width * C, C),
                                  device=y.device, dtype=torch.float32)
    else:
        out = torch.empty((B, C, height, width), device=y.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_dirfuse_fwd(
        y_c.data_ptr(), x_c.data_ptr(), _lib.dtype_code(y_c.dtype), skip.data_ptr(),
        int(skip.numel() == 4 * C), scale.data_ptr(), out.data_ptr(), int(bool(channels_last)), B,
        heads, int(height), int(width), D, _lib.stream_handle(y.device)), "vh_dirfuse_fwd")
    return out


@_lib.on_input_device
def postprocess_backward(d_out, y, x, d_skip, direction_scale, height, width):
    """Gradients of :func:`visionhope_postprocess_scale` (``vh_dirfuse_bwd``, replaces
    utils/csrc/direction_fusion.cu:123-502): d_out logical [B, C, H, W] in any layout (cast to
    fp32); y, x, d_skip, direction_scale as in the forward.  Returns (dy, dx in y's dtype and
    layout, d_skip and d_scale fp32 in the shapes of d_skip and direction_scale)."""
    g = d_out.float()
    y_c, x_c = y.contiguous(), x.contiguous()
    skip = d_skip.detach().contiguous().float()
    scale = direction_scale.detach().contiguous().float()
    B, R, heads, L, D = y_c.shape
    C = heads * D
    dy = torch.empty_like(y_c)
    dx = torch.empty_like(x_c)
    dskip = torch.empty((skip.numel(),), device=y.device, dtype=torch.float32)
    dscale = torch.empty((4, C), device=y.device, dtype=torch.float32)
    nbytes = int(_lib.load().vh_dirfuse_bwd_workspace_bytes(B, heads, int(height), int(width), D))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=y.device, dtype=torch.float32)
    sb, sc, sh, sw = g.stride()
    _lib.check(_lib.load().vh_dirfuse_bwd(
        g.data_ptr(), sb, sc, sh, sw, y_c.data_ptr(), x_c.data_ptr(), _lib.dtype_code(y_c.dtype), skip.data_ptr(),
        int(skip.numel() == 4 * C), scale.data_ptr(), dy.data_ptr(), dx.data_ptr(), dskip.data_ptr(),
        dscale.data_ptr(), ws.data_ptr(), ws.numel() * 4, B, heads, int(height), int(width), D,
        _lib.stream_handle(y.device)), "vh_dirfuse_bwd")
    return dy, dx, dskip.view(d_skip.shape), dscale.view(direction_scale.shape)


class _PostprocessFunction(torch.autograd.Function):
    """Direction restoration + fusion with its backward (utils/direction_fusion.py:84-118)."""

    @staticmethod
    def forward(ctx, y, x, d_skip, direction_scale, height, width, channels_last):
        out = _postprocess_forward(y, x, d_skip, direction_scale, height, width, channels_last)
        ctx.save_for_backward(y, x, d_skip, direction_scale)
        ctx.hw = (int(height), int(width))
        return out

    @staticmethod
    def backward(ctx, d_out):
        y, x, d_skip, scale = ctx.saved_tensors
        dy, dx, dskip, dscale = postprocess_backward(d_out, y, x, d_skip, scale, *ctx.hw)
        return dy, dx, dskip.to(d_skip.dtype), dscale.to(scale.dtype), None, None, None


def can_fuse_scale_postprocess(y, x, d_skip, direction_scale, height, width):
    if direction_scale is None:
        return False
    if not (y.is_cuda and x.is_cuda and d_skip.is_cuda and direction_scale.is_cuda):
        return False
    if any(tensor.device != y.device for tensor in (x, d_skip, direction_scale)):
        return False
    if y.dtype not in (torch.float16, torch.bfloat16, torch.float32) or x.dtype != y.dtype:
        return False
    if d_skip.dtype != torch.float32 or direction_scale.dtype != torch.float32:
        return False
    if y.dim() != 5 or x.shape != y.shape or y.shape[1] != 4:
        return False
    if tuple(d_skip.shape) not in ((y.shape[2], y.shape[4]), (4, y.shape[2], y.shape[4])):
        return False
    if tuple(direction_scale.shape) != (4, y.shape[2] * y.shape[4]):
        return False
    return int(height) * int(width) == int(y.shape[3])


def visionhope_postprocess_scale(y, x, d_skip, direction_scale, height, width, channels_last=False):
    args = (y, x, d_skip, direction_scale, int(height), int(width), bool(channels_last))
    if torch.is_grad_enabled() and any(t.requires_grad for t in (y, x, d_skip, direction_scale)):
        return _PostprocessFunction.apply(*args)
    return _postprocess_forward(*args)
