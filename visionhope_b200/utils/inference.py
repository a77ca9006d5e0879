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
    """Keep bf16 copies of a Linear / 1x1 Conv2d weight and bias on the module."""
    with torch.no_grad():
        w = _weight_2d(module).detach().to(torch.bfloat16).contiguous()
        b = None if module.bias is None else module.bias.detach().to(torch.bfloat16).contiguous()
    module._vh_half = (w, b)


def linear_cached(module, x):
    """``F.linear(x, W, b)`` for a Linear or a 1x1 Conv2d applied to channels-last rows ``x``
    (last dim = in_features), using the cached bf16 weights when x is bf16 under bf16 autocast
    with autograd off."""
    cached = getattr(module, "_vh_half", None)
    if (cached is not None and x.dtype == torch.bfloat16 and x.is_cuda and not torch.is_grad_enabled()
            and _autocast_bf16() and cached[0].device == x.device):
        return F.linear(x, cached[0], cached[1])
    return F.linear(x, _weight_2d(module), module.bias)
