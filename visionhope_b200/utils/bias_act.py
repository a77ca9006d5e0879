"""Bias and activation epilogue of a convolution whose BatchNorm was folded into it
(``vh_bias_act_fwd``): y = act(x + b) in fp32, rounded once to the requested dtype; and the
residual add with a cast (``vh_add_cast_fwd``): y = (dtype)(x + r)."""
import torch

from .. import _lib

ACTS = {None: 0, "gelu": 1}


@_lib.on_input_device
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


def add_cast_ok(x, r):
    """Whether ``add_cast`` applies: CUDA x and r of one shape, fp32/bf16, both channels-last
    contiguous (or both contiguous), with a multiple of 8 elements."""
    def dense(t):
        return t.is_contiguous(memory_format=torch.channels_last) if t.dim() == 4 else t.is_contiguous()
    return (x.is_cuda and r.device == x.device and x.shape == r.shape and x.numel() % 8 == 0
            and x.dtype in (torch.float32, torch.bfloat16) and r.dtype in (torch.float32, torch.bfloat16)
            and dense(x) and dense(r) and (x.dim() != 4 or x.stride() == r.stride()))


@_lib.on_input_device
def add_cast(x, r, out_dtype):
    """(out_dtype)(x + r), summed in fp32 and rounded once, laid out as x."""
    _lib.ensure_device(x)
    if not add_cast_ok(x, r):
        raise RuntimeError("add_cast expects dense fp32/bf16 CUDA tensors of one shape and layout")
    fmt = torch.channels_last if x.dim() == 4 else torch.contiguous_format
    y = torch.empty_like(x, dtype=out_dtype, memory_format=fmt)
    _lib.check(_lib.load().vh_add_cast_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), r.data_ptr(), _lib.dtype_code(r.dtype), y.data_ptr(),
        _lib.dtype_code(out_dtype), x.numel(), _lib.stream_handle(x.device)), "vh_add_cast_fwd")
    return y


def stem_conv_ok(x, conv):
    """Whether the first stem layer can run as ``stem_conv``: a 3-channel fp32 channels-last
    CUDA image and a 3x3 stride-2 padding-1 convolution with bias to 16/24/32/48/64 channels."""
    return (x.is_cuda and x.dim() == 4 and x.shape[1] == 3 and x.dtype == torch.float32
            and x.is_contiguous(memory_format=torch.channels_last)
            and conv.in_channels == 3 and conv.out_channels in (16, 24, 32, 48, 64) and conv.groups == 1
            and conv.kernel_size == (3, 3) and conv.stride == (2, 2) and conv.padding == (1, 1)
            and conv.dilation == (1, 1) and conv.bias is not None)


@_lib.on_input_device
def stem_conv(x, conv, act=None, out_dtype=torch.bfloat16):
    """act(bf16(conv(x)) + b) of a 3-channel channels-last fp32 image (``vh_stem_conv_fwd``):
    the first stem convolution with its folded BatchNorm and GELU.  Returns a channels-last
    tensor of ``out_dtype``."""
    _lib.ensure_device(x)
    if not stem_conv_ok(x, conv):
        raise RuntimeError("stem_conv expects a 3-channel fp32 channels-last image and a 3x3/2 convolution")
    B, _, H, W = x.shape
    cout = conv.out_channels
    w = conv.weight.detach().float().contiguous()
    b = conv.bias.detach().float().contiguous()
    y = torch.empty((B, cout, (H + 1) // 2, (W + 1) // 2), device=x.device, dtype=out_dtype,
                    memory_format=torch.channels_last)
    _lib.check(_lib.load().vh_stem_conv_fwd(
        x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), _lib.dtype_code(out_dtype), B, H, W, cout,
        ACTS[act], _lib.stream_handle(x.device)), "vh_stem_conv_fwd")
    return y
