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


def residual(res: torch.Tensor, branch: torch.Tensor, gamma: torch.Tensor, mask: torch.Tensor):
    """res + branch * gamma[c] * mask[b] over [B, C, H, W] (utils/residual.py:30-52)."""
    return res + branch * gamma.reshape(1, -1, 1, 1) * mask.reshape(-1, 1, 1, 1)


def grads(fn, inputs, grad_out):
    """fp64 CPU gradients of fn(*inputs) against grad_out, for every floating input that is a
    tensor (None for the others)."""
    leaves = [t.detach().double().cpu().requires_grad_(True) if isinstance(t, torch.Tensor) and t.is_floating_point()
              else t for t in inputs]
    out = fn(*leaves)
    out.backward(grad_out.detach().double().cpu())
    return [t.grad if isinstance(t, torch.Tensor) and t.requires_grad else None for t in leaves]


def srnl_sequence(mems, x, q, chunks, consts, q_normalized):
    """The packed SRNL recurrence (oracle/srnl_core.inc restated in PyTorch, so that autograd
    gives its gradients): mems = (M_m, M_v, M_k, e, a), shared [R, heads, D(, D)] or per chain
    [B, R, heads, D(, D)]; x [B, R, heads, L, D]; q raw [B, R, L, C] or unit-norm
    [B, R, heads, L, D]; chunks[r] the chunk length of direction r; consts = (step, min
    retention, retention bias, injection margin, spectral factor, clamp flag).  Returns y
    [B, R, heads, L, D].  Per token (models/srnl_core/csrc/inference_recurrence.cuh:40-106,
    memory.cuh:219-233), then S <- S G at each chunk end (inference_recurrence.cuh:110-135).
    The clamp limit carries the forward's one-ulp step toward zero (nextafter) in its value,
    not in its gradient."""
    step, minr, bias, margin, sfac, clamp = consts
    B, R, H, L, D = x.shape
    if not q_normalized:
        q = qnorm(q, H, D)
    per_chain = mems[0].dim() == 5
    Mm, Mv, Mk, Me, Ma = mems if per_chain else (m.unsqueeze(0).expand(B, *m.shape) for m in mems)
    eye = torch.eye(D, dtype=x.dtype)
    ys = []
    for r in range(R):
        Lc = int(chunks[r])
        n = (L + Lc - 1) // Lc
        pad = n * Lc - L
        xr = F.pad(x[:, r], (0, 0, 0, pad))
        qr = F.pad(q[:, r], (0, 0, 0, pad))
        Sm, Sv, Sk, e, a = Mm[:, r], Mv[:, r], Mk[:, r], Me[:, r], Ma[:, r]
        outs = []
        for c in range(n):
            G = eye.expand(B, H, D, D)
            for t in range(Lc):
                xt, qt = xr[:, :, c * Lc + t], qr[:, :, c * Lc + t]
                outs.append(torch.einsum("bhij,bhj->bhi", Sm, qt))
                kt = torch.einsum("bhij,bhj->bhi", Sk, xt)
                v = torch.einsum("bhij,bhj->bhi", Sv, xt)
                k = kt / torch.sqrt((kt * kt).sum(-1, keepdim=True) + 1e-6)
                d = k - v
                ep = (xt * e).sum(-1).clamp(-10.0, 10.0)
                ap = ((xt * a).sum(-1) + bias).clamp(-10.0, 10.0)
                eta = step * torch.log1p(torch.exp(ep))
                alpha = minr + (1.0 - minr) * torch.sigmoid(ap)
                dn = torch.sqrt((d * d).sum(-1) + 1e-12)
                cap = margin * (1.0 - alpha) / (dn + 1e-6)
                eff = cap * (-torch.expm1(-eta / cap))
                if clamp:
                    ke = (k * k).sum(-1)
                    lim = sfac * alpha / ke.clamp_min(1e-20)
                    lim = lim - (lim - torch.nextafter(lim.detach(), torch.zeros_like(lim))).detach()
                    eff = torch.minimum(eff, lim)
                rr = d + torch.einsum("bhij,bhj->bhi", G, k)
                G = alpha[..., None, None] * G - eff[..., None, None] * rr[..., :, None] * k[..., None, :]
            Sm, Sv, Sk = Sm @ G, Sv @ G, Sk @ G
            e = torch.einsum("bhl,bhlj->bhj", e, G)
            a = torch.einsum("bhl,bhlj->bhj", a, G)
        ys.append(torch.stack(outs, dim=2)[:, :, :L])
    return torch.stack(ys, dim=1)
