"""The four-direction scan operator of the backbone harness.

The harness (``backbone.py``) needs the VisionHOPE operator's parameters and its result, not
the reference module's path selection, autograd paths or error contract: users who want
those run the reference's own ``VisionHOPEOperator`` over this package's drop-in modules.
So this module is small and built around the one launch the harness makes:

* ``ScanMemories`` owns the five initial memories of the four scans.  Their names and
  shapes are the reference's (``models/srnl.py:55-61``: ``M_m_0, M_v_0, M_k_0`` are
  ``[4, heads, D, D]``, ``M_eta_0, M_alpha_0`` are ``[4, heads, D]``), so a reference
  ``state_dict`` loads; the initialisation follows ``models/srnl.py:70-74``.
* ``ScanMixer`` owns ``W_q``, the per-head skip and the direction weights (names and shapes of
  ``models/operator.py:36-47``) and computes, for a channels-last ``x``, the operator's output
  ``sum_d w_d (y_d + s_d x)`` in image order with one ``vh_srnl_spatial_fwd`` launch on the
  image and its single ``W_q`` projection (the kernel applies each scan's index map while
  loading; nothing is serialized).  Under autocast the queries are projected in the autocast
  dtype and the scan runs in that dtype when ``x`` has it (the reference's fast path); an
  ``x`` of another dtype has its queries converted to its own dtype first.

Image-aligned chunks only (rows of W tokens, columns of H tokens: the ``chunk_size=None`` of
every VisionHOPE model configuration); a fixed chunk length is rejected.
"""
from __future__ import annotations

import torch
from torch import nn

from .srnl_core.fused import spatial_forward
from .utils.inference import linear_cached

_MERGES = ("sum", "scale", "softmax")


class ScanMemories(nn.Module):
    """Initial memories of the four directional scans of one operator (fp32 parameters)."""

    def __init__(self, dim: int, head_dim: int = 16, directions: int = 4):
        super().__init__()
        if dim <= 0 or head_dim <= 0 or dim % head_dim:
            raise ValueError("dim must be a positive multiple of head_dim")
        self.head_dim = head_dim
        self.num_heads = dim // head_dim
        lead = (directions, self.num_heads)
        for name in ("M_m_0", "M_v_0", "M_k_0"):
            setattr(self, name, nn.Parameter(torch.empty(*lead, head_dim, head_dim)))
        for name in ("M_eta_0", "M_alpha_0"):
            setattr(self, name, nn.Parameter(torch.empty(*lead, head_dim)))
        self.reset_parameters()

    @property
    def initial_memories(self):
        return self.M_m_0, self.M_v_0, self.M_k_0, self.M_eta_0, self.M_alpha_0

    @torch.no_grad()
    def reset_parameters(self):
        for m in self.initial_memories[:3]:
            nn.init.trunc_normal_(m, std=0.01, a=-2.0, b=2.0)
        for v in self.initial_memories[3:]:
            v.zero_()

    @torch.no_grad()
    def densify(self):
        """Store the matrices dense: the kernel reads them as contiguous fp32, and a model
        converted to channels_last holds these 4-D parameters permuted."""
        for m in self.initial_memories:
            if not m.is_contiguous():
                m.data = m.data.contiguous()


class ScanMixer(nn.Module):
    """``out[b, h, w, c] = sum_d w_d[c] (y_d + s_d x)[b, h, w, c]`` over the four scans."""

    def __init__(self, dim: int, head_dim: int = 16, direction_merge: str = "scale",
                 share_direction_skip: bool = True):
        super().__init__()
        if direction_merge not in _MERGES:
            raise ValueError(f"direction_merge must be one of {_MERGES}")
        self.dim, self.head_dim = int(dim), int(head_dim)
        self.direction_merge = direction_merge
        self.srnl = ScanMemories(dim, head_dim)
        self.num_heads = self.srnl.num_heads
        self.W_q = nn.Linear(dim, dim)
        skip = (self.num_heads, head_dim) if share_direction_skip else (4, self.num_heads, head_dim)
        self.d_skip = nn.Parameter(torch.zeros(skip))
        self.direction_scale = nn.Parameter(torch.ones(4, dim)) if direction_merge == "scale" else None
        self.direction_logits = nn.Parameter(torch.zeros(4, dim)) if direction_merge == "softmax" else None
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        self.srnl.reset_parameters()
        nn.init.trunc_normal_(self.W_q.weight, std=0.02, a=-2.0, b=2.0)
        self.W_q.bias.zero_()
        self.d_skip.zero_()
        if self.direction_scale is not None:
            self.direction_scale.fill_(1.0)
        if self.direction_logits is not None:
            self.direction_logits.zero_()

    def fusion_weights(self) -> torch.Tensor:
        """The per-direction channel weights w_d as fp32 [4, C] (models/operator.py:72-77)."""
        if self.direction_merge == "scale":
            return self.direction_scale.detach().float()
        if self.direction_merge == "softmax":
            return 4.0 * torch.softmax(self.direction_logits.detach().float(), dim=0)
        return torch.ones(4, self.dim, device=self.d_skip.device)

    def forward(self, x: torch.Tensor, *, addend: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """x: [B, C, H, W] on a CUDA device (any memory format; channels-last avoids a copy).
        Returns NHWC [B, H, W, C]: fp32, or, with ``out_dtype``, ``(out_dtype)(out + addend)``
        written by the scan launch itself (``addend`` NHWC in the scan's dtype, or None)."""
        if x.ndim != 4 or x.shape[1] != self.dim or min(x.shape) <= 0:
            raise ValueError(f"ScanMixer expects a nonempty [B, {self.dim}, H, W] tensor")
        if not x.is_cuda:
            raise RuntimeError("ScanMixer runs on CUDA tensors only")
        height, width = int(x.shape[2]), int(x.shape[3])
        img = x.permute(0, 2, 3, 1)
        if not img.is_contiguous():
            img = img.contiguous()
        q = linear_cached(self.W_q, img)
        if q.dtype != img.dtype:
            q = q.to(img.dtype)
        if addend is not None and addend.dtype != img.dtype:
            addend = addend.to(img.dtype)
        return spatial_forward(self.srnl.initial_memories, img, q, self.d_skip, self.fusion_weights(),
                               height, width, self.head_dim, layout="image", addend=addend,
                               final_dtype=out_dtype)
