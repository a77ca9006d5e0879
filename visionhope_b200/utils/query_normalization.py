"""Fused query normalization and layout conversion (mirror of utils/query_normalization.py).

``visionhope_qnorm(q_raw [B, 4, L, C], heads, D)`` -> fp32 [B, 4, heads, L, D], computed by
``vh_qnorm_fwd`` (replaces utils/csrc/query_normalization.cu:136-178); the autograd path runs
``vh_qnorm_bwd`` (query_normalization.cu:78-134).
"""
import torch

from .. import _lib


@_lib.on_input_device
def _qnorm_forward(q_raw, num_heads, head_dim, want_inv=False):
    _lib.ensure_device(q_raw)
    q = q_raw.contiguous()
    if q.dim() != 4 or q.shape[1] != 4 or q.shape[3] != num_heads * head_dim:
        raise RuntimeError("Invalid QRaw shape for visionhope_qnorm_forward.")
    B, R, L, _ = q.shape
    out = torch.empty((B, R, num_heads, L, head_dim), device=q.device, dtype=torch.float32)
    inv = torch.empty((B * R * L * num_heads,), device=q.device, dtype=torch.float32) if want_inv else None
    _lib.check(_lib.load().vh_qnorm_fwd(q.data_ptr(), _lib.dtype_code(q.dtype), out.data_ptr(), _lib.ptr(inv),
                                        B, R, L, num_heads, head_dim, _lib.stream_handle(q.device)),
               "vh_qnorm_fwd")
    return (out, inv) if want_inv else out


@_lib.on_input_device
def qnorm_backward(grad_out, q_out, inv_norm, num_heads, head_dim, q_dtype):
    """Gradient of :func:`visionhope_qnorm` (``vh_qnorm_bwd``, replaces
    utils/csrc/query_normalization.cu:78-134): grad_out [B, 4, heads, L, D] (cast to fp32), the
    forward's output and 1/norm; returns d q_raw [B, 4, L, C] in q_raw's dtype."""
    g = grad_out.contiguous().float()
    B, R, heads, L, D = q_out.shape
    dq = torch.empty((B, R, L, heads * D), device=q_out.device, dtype=q_dtype)
    _lib.check(_lib.load().vh_qnorm_bwd(g.data_ptr(), q_out.data_ptr(), inv_norm.data_ptr(), dq.data_ptr(),
                                        _lib.dtype_code(q_dtype), B, R, L, heads, D,
                                        _lib.stream_handle(q_out.device)), "vh_qnorm_bwd")
    return dq


class _QNormFunction(torch.autograd.Function):
    """Query normalization with its backward (utils/query_normalization.py:53-76)."""

    @staticmethod
    def forward(ctx, q_raw, num_heads, head_dim):
        out, inv = _qnorm_forward(q_raw, num_heads, head_dim, want_inv=True)
        ctx.save_for_backward(out, inv)
        ctx.meta = (int(num_heads), int(head_dim), q_raw.dtype)
        return out

    @staticmethod
    def backward(ctx, grad):
        out, inv = ctx.saved_tensors
        heads, D, dtype = ctx.meta
        return qnorm_backward(grad, out, inv, heads, D, dtype), None, None


def can_fuse_qnorm(q_raw, num_heads, head_dim):
    if not q_raw.is_cuda or q_raw.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return False
    if q_raw.dim() != 4 or q_raw.shape[1] != 4:
        return False
    if int(head_dim) not in {4, 8, 16, 32, 64}:
        return False
    return int(q_raw.shape[-1]) == int(num_heads) * int(head_dim)


def visionhope_qnorm(q_raw, num_heads, head_dim):
    if torch.is_grad_enabled() and q_raw.requires_grad:
        return _QNormFunction.apply(q_raw, int(num_heads), int(head_dim))
    return _qnorm_forward(q_raw, int(num_heads), int(head_dim))
