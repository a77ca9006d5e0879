"""LayerScale residual add of the block with drop path (mirror of utils/residual.py).

``visionhope_residual_add`` and ``can_fuse_residual_add`` keep the reference's names, arguments
and results: the output is fp32 channels-last ``residual + branch * gamma * mask``, where mask
is the per-sample drop-path keep mask (divided by the keep probability when scale_by_keep),
drawn with the same ``bernoulli_`` call so that a seeded generator gives the same mask.  The
reference's Triton kernels are replaced by ``vh_residual_add_fwd`` (residual.py:30-52) and
``vh_residual_add_bwd`` (residual.py:54-101).
"""
import torch

from .. import _lib


@_lib.on_input_device
def residual_add_forward(residual, branch, gamma, mask):
    """fp32 channels-last residual + branch * gamma[c] * mask[b] (``vh_residual_add_fwd``)."""
    _lib.ensure_device(branch)
    if residual.shape != branch.shape or branch.dim() != 4:
        raise RuntimeError("visionhope_residual_add expects residual and branch of one [B, C, H, W] shape")
    residual = residual.contiguous(memory_format=torch.channels_last)  # no copy when already so
    branch = branch.contiguous(memory_format=torch.channels_last)
    batch, channels, height, width = branch.shape
    out = torch.empty_like(branch, dtype=torch.float32, memory_format=torch.channels_last)
    g = gamma.detach().reshape(-1).contiguous().float()
    m = mask.detach().reshape(-1).contiguous().float()
    _lib.check(_lib.load().vh_residual_add_fwd(
        residual.data_ptr(), _lib.dtype_code(residual.dtype), branch.data_ptr(), _lib.dtype_code(branch.dtype),
        g.data_ptr(), m.data_ptr(), out.data_ptr(), batch, height * width, channels,
        _lib.stream_handle(branch.device)), "vh_residual_add_fwd")
    return out


@_lib.on_input_device
def residual_add_backward(dout, branch, gamma, mask):
    """(d branch in branch's dtype, channels-last; d gamma fp32 [C]) (``vh_residual_add_bwd``);
    d residual is dout itself."""
    batch, channels, height, width = branch.shape
    branch = branch.contiguous(memory_format=torch.channels_last)
    d = dout.contiguous(memory_format=torch.channels_last).float()
    g = gamma.detach().reshape(-1).contiguous().float()
    m = mask.detach().reshape(-1).contiguous().float()
    dbranch = torch.empty_like(branch, memory_format=torch.channels_last)
    dgamma = torch.empty((channels,), device=branch.device, dtype=torch.float32)
    rows = batch * height * width
    nbytes = int(_lib.load().vh_residual_add_bwd_workspace_bytes(rows, channels))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=branch.device, dtype=torch.float32)
    _lib.check(_lib.load().vh_residual_add_bwd(
        d.data_ptr(), branch.data_ptr(), _lib.dtype_code(branch.dtype), g.data_ptr(), m.data_ptr(),
        dbranch.data_ptr(), dgamma.data_ptr(), ws.data_ptr(), ws.numel() * 4, batch, height * width, channels,
        _lib.stream_handle(branch.device)), "vh_residual_add_bwd")
    return dbranch, dgamma


class _VisionHOPEResidualFunction(torch.autograd.Function):
    """residual.py:104-169: saves branch, gamma and the mask; d residual = d out."""

    @staticmethod
    def forward(ctx, residual, branch, gamma, mask):
        out = residual_add_forward(residual, branch, gamma, mask)
        ctx.save_for_backward(branch, gamma, mask)
        return out

    @staticmethod
    def backward(ctx, dout):
        branch, gamma, mask = ctx.saved_tensors
        dout = dout.contiguous(memory_format=torch.channels_last)
        dbranch, dgamma = residual_add_backward(dout, branch, gamma, mask)
        return dout, dbranch, dgamma.view(gamma.shape).to(gamma.dtype), None


def can_fuse_residual_add(residual, branch, gamma):
    """residual.py:172-192 without its Triton row-capacity limit (the CUDA kernels take any C)."""
    if residual.ndim != 4 or branch.ndim != 4 or residual.shape != branch.shape:
        return False
    if not residual.is_cuda or not branch.is_cuda or not gamma.is_cuda:
        return False
    if residual.device != branch.device or gamma.device != branch.device:
        return False
    if not gamma.is_contiguous() or not gamma.is_floating_point():
        return False
    if not residual.is_contiguous(memory_format=torch.channels_last):
        return False
    if not branch.is_contiguous(memory_format=torch.channels_last):
        return False
    if (branch.dtype not in (torch.float16, torch.bfloat16, torch.float32)
            or residual.dtype not in (torch.float16, torch.bfloat16, torch.float32)):
        return False
    channels = branch.shape[1]
    return gamma.numel() == channels and channels > 0


def visionhope_residual_add(residual, branch, gamma, drop_prob, training, scale_by_keep=True):
    """residual.py:195-204: the drop-path mask (ones outside training), then the fused add."""
    batch = branch.shape[0]
    if training and drop_prob > 0.0:
        keep_prob = 1.0 - float(drop_prob)
        mask = torch.empty((batch,), device=branch.device, dtype=torch.float32).bernoulli_(keep_prob)
        if keep_prob > 0.0 and scale_by_keep:
            mask.div_(keep_prob)
    else:
        mask = torch.ones((batch,), device=branch.device, dtype=torch.float32)
    return _VisionHOPEResidualFunction.apply(residual, branch, gamma, mask)
