"""Fused query normalization and layout conversion (mirror of utils/query_normalization.py).

``visionhope_qnorm(q_raw [B, 4, L, C], heads, D)`` -> fp32 [B, 4, heads, L, D], computed by
``vh_qnorm_fwd`` (replaces utils/csrc/query_normalization.cu:136-178).  Forward only.
"""
import torch

from .. import _lib


@_lib.on_input_device
def _qnorm_forward(q_raw, num_heads, head_dim):
    _lib.ensure_device(q_raw)
    q = q_raw.contiguous()
    if q.dim() != 4 or q.shape[1] != 4 or q.shape[3] != num_heads * head_dim:
        raise RuntimeError("Invalid QRaw shape for visionhope_qnorm_forward.")
    B, R, L, _ = q.shape
    out = torch.empty((B, R, num_heads, L, head_dim), device=q.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_qnorm_fwd(q.data_ptr(), _lib.dtype_code(q.dtype), out.data_ptr(), None,
                                        B, R, L, num_heads, head_dim, _lib.stream_handle(q.device)),
               "vh_qnorm_fwd")
    return out


class _QNormForwardOnly(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q_raw, num_heads, head_dim):
        return _qnorm_forward(q_raw, num_heads, head_dim)

    @staticmethod
    def backward(ctx, grad):
        raise NotImplementedError("query-normalization backward is not implemented by visionhope_b200")


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
        return _QNormForwardOnly.apply(q_raw, int(num_heads), int(head_dim))
    return _qnorm_forward(q_raw, int(num_heads), int(head_dim))
