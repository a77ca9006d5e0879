"""Depthwise convolutions of the VisionHOPE block with their elementwise epilogues fused
(``vh_dwconv_fwd``): one pass over HBM instead of a convolution, a bias pass and the
activation / gate / residual passes that follow it in models/block.py and the FFN.

Inference only (no autograd); channels-last CUDA tensors of fp32 or bf16.
"""
import torch

from .. import _lib

MODES = {"bias": 0, "resid": 1, "gate": 2, "gelu": 3, "resid_add": 4, "gate_pos": 5}


def fusable(x, conv):
    """Whether ``conv`` applied to ``x`` can run as a fused depthwise call: a depthwise
    3/5/7 stride-1 'same' convolution with bias of a channels-last fp32/bf16 CUDA tensor whose
    channel count is a multiple of 8, with autograd off and bf16 autocast on (the kernel's
    arithmetic is that of a bf16 convolution)."""
    k = conv.kernel_size[0]
    return (x.is_cuda and x.dim() == 4 and not torch.is_grad_enabled()
            and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
            and x.dtype in (torch.float32, torch.bfloat16)
            and x.is_contiguous(memory_format=torch.channels_last) and x.shape[1] % 8 == 0
            and conv.groups == conv.in_channels == conv.out_channels == x.shape[1]
            and conv.kernel_size == (k, k) and k in (3, 5, 7) and conv.stride == (1, 1)
            and conv.padding == (k // 2, k // 2) and conv.dilation == (1, 1) and conv.bias is not None)


def gate_pos_ok(x, conv, pos_conv):
    """Whether the gated 7x7 ``conv`` and the 5x5 ``pos_conv`` on its output can run as one
    "gate_pos" call: both fusable, bf16, and whole 14 x 14 or 7 x 7 images (one CTA holds an
    image, so the second convolution reads the first one's output from shared memory)."""
    H, W = x.shape[-2:]
    return (x.dtype == torch.bfloat16 and (H, W) in ((14, 14), (7, 7)) and conv.kernel_size == (7, 7)
            and pos_conv.kernel_size == (5, 5) and fusable(x, conv) and fusable(x, pos_conv))


@_lib.on_input_device
def depthwise_fused(x, conv, mode, gate=None, addend=None, with_sumsq=False, pos_conv=None):
    """Apply depthwise ``conv`` to channels-last NCHW ``x`` with epilogue ``mode``:
    "bias": conv(x) + b;  "resid": s + (conv(s) + b) with s = x, or s = x + addend when an
    addend (fp32/bf16, x's shape) is given;  "gate": x + sigmoid(gate) * (conv(x) + b);
    "gelu": h = gelu(x), gelu(h + conv(h) + b);  "gate_pos": y as "gate", and also
    pos_conv(y) + pos_b (see ``gate_pos_ok``), returned as a second tensor.  Returns a
    channels-last tensor of x's dtype, and with ``with_sumsq`` ("gelu" only) also the fp32
    [B, tiles, C] sums of y^2 per pixel tile that a following GRN needs
    (``grn_cuda.grn_apply``)."""
    _lib.ensure_device(x)
    B, C, H, W = x.shape
    if mode not in MODES:
        raise ValueError(f"unknown depthwise epilogue {mode!r}")
    gate_dtype = 0
    if mode == "gate_pos" and (pos_conv is None or not gate_pos_ok(x, conv, pos_conv)):
        raise RuntimeError("gate_pos needs bf16 14x14 or 7x7 images, a 7x7 conv and a 5x5 pos_conv")
    if mode in ("gate", "gate_pos"):
        if gate is None or gate.shape != x.shape or gate.dtype != x.dtype:
            raise RuntimeError("the gated epilogue needs a gate of x's shape and dtype")
        gate = gate.contiguous(memory_format=torch.channels_last)
    if addend is not None:
        if mode != "resid" or addend.shape != x.shape or addend.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("an addend goes with the residual epilogue, fp32/bf16 of x's shape")
        mode, gate = "resid_add", addend.contiguous(memory_format=torch.channels_last)
        gate_dtype = _lib.dtype_code(gate.dtype)
    x = x.contiguous(memory_format=torch.channels_last)
    w = conv.weight.detach().float().contiguous()
    b = conv.bias.detach().float().contiguous()
    y = torch.empty_like(x, memory_format=torch.channels_last)
    sumsq = None
    if with_sumsq:
        if mode != "gelu":
            raise RuntimeError("tile statistics go with the gelu epilogue")
        sumsq = torch.empty((B, int(_lib.load().vh_dwconv_tiles(H, W)), C), device=x.device, dtype=torch.float32)
    pw = pb = pos = None
    if mode == "gate_pos":
        pw = pos_conv.weight.detach().float().contiguous()
        pb = pos_conv.bias.detach().float().contiguous()
        pos = torch.empty_like(x, memory_format=torch.channels_last)
    args = _lib.VhDwconvArgs(x.data_ptr(), _lib.ptr(gate), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                             _lib.dtype_code(x.dtype), MODES[mode], conv.kernel_size[0], B, H, W, C, gate_dtype,
                             _lib.ptr(sumsq), _lib.ptr(pw), _lib.ptr(pb), _lib.ptr(pos),
                             5 if mode == "gate_pos" else 0)
    _lib.check(_lib.load().vh_dwconv_fwd(args, _lib.stream_handle(x.device)), "vh_dwconv_fwd")
    if mode == "gate_pos":
        return y, pos
    return (y, sumsq) if with_sumsq else y
