"""Gradient oracle: the forward formulas of the path restated in plain PyTorch, run in fp64 on
the CPU, whose autograd gradients are what the backward kernels are checked against.

TEST INFRASTRUCTURE ONLY: nothing in the product imports or runs this file.  Each function
cites the reference code whose forward it restates; the gradients follow from autograd, so
they are exact (to fp64) for the restated forward.  The forwards themselves are pinned in
tests/test_oracle_grad.py: against the C oracle (vhope_oracle.c, itself pinned against the
reference's kernels) and against the reference's own CPU code (grn_reference, F.layer_norm).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def qnorm(q_raw: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """q_raw [B, R, L, C] -> [B, R, heads, L, D] = q / max(||q||, 1e-12) per head vector
    (utils/csrc/query_normalization.cu:136-178)."""
    B, R, L, _ = q_raw.shape
    q = q_raw.reshape(B, R, L, heads, head_dim).permute(0, 1, 3, 2, 4)
    return q / q.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def scan_positions(H: int, W: int) -> torch.Tensor:
    """[4, L]: the position in scan d of each row-major pixel (models/operator.py:79-86)."""
    L = H * W
    pix = torch.arange(L)
    i, j = pix // W, pix % W
    col = j * H + i
    return torch.stack([pix, L - 1 - pix, col, L - 1 - col])


def dirfuse(y: torch.Tensor, x: torch.Tensor, skip: torch.Tensor, scale: torch.Tensor, H: int, W: int):
    """y, x [B, 4, heads, L, D]; skip C or [4, C]; scale [4, C] -> out [B, C, H, W] =
    sum_d scale[d] (y_d + skip_d x_d) restored to image order (utils/csrc/direction_fusion.cu:11-65)."""
    B, R, heads, L, D = y.shape
    C = heads * D
    pos = scan_positions(H, W)
    sk = skip.reshape(-1, C)
    if sk.shape[0] == 1:
        sk = sk.expand(4, C)
    out = 0
    for d in range(4):
        yd = y[:, d].permute(0, 2, 1, 3).reshape(B, L, C)[:, pos[d]]  # [B, L(pixels), C]
        xd = x[:, d].permute(0, 2, 1, 3).reshape(B, L, C)[:, pos[d]]
        out = out + scale[d] * (yd + sk[d] * xd)
    return out.reshape(B, H, W, C).permute(0, 3, 1, 2)


def layernorm_rows(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float):
    """LayerNorm over the last axis (utils/layer_norm_cuda.py:31-57, models/layers.py:17-35)."""
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def grn(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float):
    """x [B, C, H, W] -> x (1 + gamma Gx / (mean_c Gx + eps)) + beta, Gx = ||x||_2 over H, W
    (utils/grn.py:26-38, utils/csrc/grn_cuda.cu:46-124)."""
    gx = x.pow(2).sum(dim=(2, 3), keepdim=True).sqrt()
    nx = gx / (gx.mean(dim=1, keepdim=True) + eps)
    return x * (1 + gamma.reshape(1, -1, 1, 1) * nx) + beta.reshape(1, -1, 1, 1)


def grads(fn, inputs, grad_out):
    """fp64 CPU gradients of fn(*inputs) against grad_out, for every floating input that is a
    tensor (None for the others)."""
    leaves = [t.detach().double().cpu().requires_grad_(True) if isinstance(t, torch.Tensor) and t.is_floating_point()
              else t for t in inputs]
    out = fn(*leaves)
    out.backward(grad_out.detach().double().cpu())
    return [t.grad if isinstance(t, torch.Tensor) and t.requires_grad else None for t in leaves]
