"""Global Response Normalization (mirror of utils/grn.py), fp32 output.

    y = x * (1 + gamma * Gx / (mean_c Gx + eps)) + beta,   Gx[b, c] = ||x[b, c, :, :]||_2

Every CUDA input runs on ``vh_grn_fwd``; inputs not stored channels-last are converted
first.  There is no CPU path: CPU tensors raise.  ``grn_reference`` is the reference's
formula (utils/grn.py:26-38) kept for API completeness; no product path calls it.
"""
import torch
from torch import nn

from .grn_cuda import visionhope_grn

__all__ = ["GlobalResponseNorm", "global_response_norm", "grn_reference"]


def _check_shape(x, gamma, beta):
    if x.ndim != 4:
        raise ValueError("GRN expects logical NCHW input with four dimensions")
    if not x.is_floating_point() or not gamma.is_floating_point() or not beta.is_floating_point():
        raise TypeError("GRN expects floating-point input and channel parameters")
    if gamma.numel() != x.shape[1] or beta.numel() != x.shape[1]:
        raise ValueError("GRN gamma and beta must each contain one value per channel")
    if gamma.device != x.device or beta.device != x.device:
        raise ValueError("GRN input, gamma and beta must be on the same device")


def grn_reference(x, gamma, beta, eps=1e-6):
    """The GRN formula in PyTorch fp32 (utils/grn.py:26-38); not used by any product path."""
    _check_shape(x, gamma, beta)
    x = x.float()
    gamma = gamma.float().reshape(1, x.shape[1], 1, 1)
    beta = beta.float().reshape(1, x.shape[1], 1, 1)
    gx = torch.norm(x, p=2, dim=(2, 3), keepdim=True)
    nx = gx / (gx.mean(dim=1, keepdim=True) + float(eps))
    return x * (1.0 + gamma * nx) + beta


def global_response_norm(x, gamma, beta, eps=1e-6):
    """fp32 GRN on the B200 kernel (channels-last storage; other layouts are converted)."""
    _check_shape(x, gamma, beta)
    if not x.is_cuda:
        raise RuntimeError("global_response_norm runs on CUDA only (visionhope_b200 has no CPU path)")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        x = x.float()
    if not x.is_contiguous(memory_format=torch.channels_last):
        x = x.contiguous(memory_format=torch.channels_last)
    return visionhope_grn(x, gamma.float(), beta.float(), float(eps))


class GlobalResponseNorm(nn.Module):
    """GRN for logical NCHW tensors, with FP32 output (utils/grn.py:54-70)."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.gamma = nn.Parameter(torch.zeros(1, dim, 1, 1, dtype=torch.float32))
        self.beta = nn.Parameter(torch.zeros(1, dim, 1, 1, dtype=torch.float32))
        self.eps = float(eps)

    def forward(self, x):
        return global_response_norm(x, self.gamma, self.beta, self.eps)

    def extra_repr(self):
        return f"dim={self.gamma.numel()}, eps={self.eps}, output_dtype=float32"
