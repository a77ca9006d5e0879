"""Bias and activation epilogue of a convolution whose BatchNorm was folded into it
(``vh_bias_act_fwd``): y = act(x + b) in fp32, rounded once to the requested dtype."""
import torch

from .. import _lib
from .cuda import on_tensor_device

ACTS = {None: 0, "gelu": 1}


@on_tensor_device
def bias_act(x, bias, act=None, out_dtype=None):
    """x: channels-last NCHW CUDA tensor (C a multiple of 8); bias: [C].  Returns a channels-last
    tensor of ``out_dtype`` (default x's dtype)."""
    _lib.ensure_device(x)
    B, C, H, W = x.shape
    x = x.contiguous(memory_format=torch.channels_last)
    b = bias.detach().float().contiguous()
    out_dtype = out_dtype or x.dtype
    y = torch.empty_like(x, dtype=out_dtype, memory_format=torch.channels_last)
    _lib.check(_lib.load().vh_bias_act_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), b.data_ptr(), y.data_ptr(), _lib.dtype_code(out_dtype),
        B * H * W, C, ACTS[act], _lib.stream_handle(x.device)), "vh_bias_act_fwd")
    return y
