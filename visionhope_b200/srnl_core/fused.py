"""Inference-only execution for spatial scans and general SRNL sequences (libvhope.so).

Mirror of models/srnl_core/fused.py: ``load_fused_cuda(io_dtype)`` returns an object that
exposes the reference extension's functions (fused.cpp:1-61, fused.cu:131-351) with the
same arguments and results, and ``srnl_sequence_inference`` keeps its signature.  The
"atomic" and "noatomic" variants are one implementation here: the fused kernel writes each
pixel in a fixed order, so every variant is deterministic and allocates only its output.
"""
from __future__ import annotations

import torch

from .. import _lib
from .chunk import SUPPORTED_HEAD_DIMS, recurrence_constants, run_sequence


def _f32(t, device):
    return t.detach().contiguous().to(device=device, dtype=torch.float32)


def spatial_forward(states, x, q, d_skip, weights, height, width, head_dim, *, layout,
                    out=None, concurrent=True, addend=None, final_dtype=None):
    """Fused four-scan operator; returns fp32 [B, H, W, C] (or final_dtype, see below).

    layout "scans":  x, q are the four serialized scans [B, 4, L, C].
    layout "packed": x is [B, 4, heads, L, D], q is [B, 4, L, C].
    layout "image":  x, q are one channels-last image each ([B, H, W, C] or any tensor whose
                     pixel p / channel c element sits at b*sB + p*sP + c); scans are index maps.
    concurrent:      give the library three fp32 workspace planes so the four scans run in one
                     launch, each into its own plane (used where the warp-per-chain scan
                     applies).
    final_dtype:     return a new [B, H, W, C] tensor of this dtype holding the sum plus
                     `addend` (x's dtype, [B, H, W, C] with unit channel stride), written by the
                     scan launch itself when it runs concurrently; `out` is then scratch.
    """
    _lib.ensure_device(x)
    H, W, D = int(height), int(width), int(head_dim)
    if D not in SUPPORTED_HEAD_DIMS:
        raise RuntimeError("line fused HOPE supports head_dim in {4, 8, 16, 32, 64}.")
    if x.dtype != q.dtype:
        raise RuntimeError("line fused HOPE forward expects matching X and Q_raw dtypes.")
    dev = x.device
    mems = tuple(_f32(s, dev) for s in states)
    skip = _f32(d_skip, dev)
    wts = _f32(weights, dev)
    B = int(x.shape[0])
    L = H * W
    if layout == "scans":
        x = x.contiguous()
        q = q.contiguous()
        C = int(x.shape[3])
        if tuple(x.shape) != (B, 4, L, C) or tuple(q.shape) != (B, 4, L, C):
            raise RuntimeError("line fused seq-layout HOPE got inconsistent H/W, C, and head_dim.")
        xs = (4 * L * C, L * C, C, D)
        qs = (4 * L * C, L * C, C, D)
        remap = 0
    elif layout == "packed":
        x = x.contiguous()
        q = q.contiguous()
        heads = int(x.shape[2])
        C = heads * D
        if tuple(x.shape) != (B, 4, heads, L, D) or tuple(q.shape) != (B, 4, L, C):
            raise RuntimeError("line fused HOPE got inconsistent H/W and sequence length.")
        xs = (4 * heads * L * D, heads * L * D, D, L * D)
        qs = (4 * L * C, L * C, C, D)
        remap = 0
    elif layout == "image":
        C = int(x.shape[-1])
        x = x.reshape(B, L, C)
        q = q.reshape(B, L, C)
        if x.stride(2) != 1 or q.stride(2) != 1:
            x = x.contiguous()
            q = q.contiguous()
        xs = (x.stride(0), 0, x.stride(1), D)
        qs = (q.stride(0), 0, q.stride(1), D)
        remap = 1
    else:
        raise ValueError(f"unknown layout {layout!r}")
    heads = C // D
    if heads * D != C:
        raise RuntimeError("line fused seq-layout HOPE got inconsistent H/W, C, and head_dim.")
    if skip.numel() not in (C, 4 * C):
        raise RuntimeError("d_skip must contain C or 4*C values")
    if tuple(wts.shape) != (4, C):
        raise RuntimeError("direction weights must be fp32 [4, C]")
    if out is None:
        out = torch.empty((B, H, W, C), device=dev, dtype=torch.float32)
    aux = torch.empty(3 * B * out.stride(0), device=dev, dtype=torch.float32) if concurrent else None
    final = None
    if final_dtype is not None:
        final = torch.empty((B, H, W, C), device=dev, dtype=final_dtype)
    if addend is not None:
        if final is None:
            raise RuntimeError("an addend requires final_dtype")
        if addend.dtype != x.dtype or addend.device != dev:
            raise RuntimeError("the addend must match x's dtype and device")
        addend = addend.reshape(B, L, C)
        if addend.stride(2) != 1 or addend.stride(1) != C:
            addend = addend.contiguous()
    args = _lib.VhSpatialArgs(
        _lib.memories(mems), x.data_ptr(), q.data_ptr(), *xs, *qs, _lib.dtype_code(x.dtype), remap,
        skip.data_ptr(), int(skip.numel() == 4 * C), wts.data_ptr(), out.data_ptr(),
        out.stride(0), B, H, W, heads, D, recurrence_constants(),
        aux.data_ptr() if aux is not None else None,
        addend.data_ptr() if addend is not None else None,
        addend.stride(0) if addend is not None else 0,
        final.data_ptr() if final is not None else None,
        _lib.dtype_code(final_dtype) if final is not None else 0,
        final.stride(0) if final is not None else 0)
    _lib.check(_lib.load().vh_srnl_spatial_fwd(args, _lib.stream_handle(dev)), "vh_srnl_spatial_fwd")
    return final if final is not None else out


class _FusedModule:
    """The functions of the reference's fused extension for one I/O dtype."""

    def __init__(self, io_dtype):
        self.io_dtype = io_dtype

    def _check(self, X, Q_raw, M_m_0, D_skip, Dir_weight):
        if X.dtype != self.io_dtype or Q_raw.dtype != self.io_dtype:
            raise RuntimeError(f"line fused HOPE forward expects {self.io_dtype} X and Q_raw.")
        if M_m_0.dtype != torch.float32 or D_skip.dtype != torch.float32 or Dir_weight.dtype != torch.float32:
            raise RuntimeError("line fused HOPE forward expects fp32 state, skip, and direction weights.")

    @_lib.on_input_device
    def srnl_line_forward_seq_noatomic(self, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, X, Q_raw,
                                       D_skip, Dir_weight, H, W, D_int):
        """X, Q_raw [B, 4, L, C] -> fp32 [B, H, W, C] (fused.cu:307-351)."""
        self._check(X, Q_raw, M_m_0, D_skip, Dir_weight)
        return spatial_forward((M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0), X, Q_raw, D_skip,
                               Dir_weight, H, W, D_int, layout="scans")

    srnl_line_forward_seq = srnl_line_forward_seq_noatomic

    @_lib.on_input_device
    def srnl_line_forward_noatomic(self, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, X, Q_raw,
                                   D_skip, Dir_weight, H, W, D_int):
        """X packed [B, 4, heads, L, D], Q_raw [B, 4, L, C] -> fp32 [B, H, W, C] (fused.cu:221-262)."""
        self._check(X, Q_raw, M_m_0, D_skip, Dir_weight)
        return spatial_forward((M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0), X, Q_raw, D_skip,
                               Dir_weight, H, W, D_int, layout="packed")

    srnl_line_forward = srnl_line_forward_noatomic

    @_lib.on_input_device
    def srnl_sequence_forward(self, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, X, Q_raw, chunk_sizes):
        """X [B, R, heads, N, D], Q_raw [B, R, N, C] -> [B, R, heads, N, D] in X's dtype."""
        if not (X.is_cuda and X.dim() == 5):
            raise RuntimeError("SRNL inference expects contiguous CUDA [B, directions, heads, N, d]")
        if X.dtype != self.io_dtype or Q_raw.dtype != X.dtype or Q_raw.device != X.device:
            raise RuntimeError("SRNL inference requires matching input/query dtype and device")
        B, R, heads, length, D = X.shape
        if not (B > 0 and heads > 0 and length > 0 and R in (1, 2, 4)):
            raise RuntimeError("SRNL inference requires nonempty inputs and 1, 2, or 4 directions")
        if D not in SUPPORTED_HEAD_DIMS:
            raise RuntimeError("Unsupported SRNL head dimension")
        if tuple(Q_raw.shape) != (B, R, length, heads * D):
            raise RuntimeError("Invalid raw query shape")
        for s in (M_m_0, M_v_0, M_k_0):
            if s.dtype != torch.float32 or tuple(s.shape) != (R, heads, D, D):
                raise RuntimeError("SRNL matrix memories must be contiguous FP32 [directions, heads, d, d]")
        for s in (M_eta_0, M_alpha_0):
            if s.dtype != torch.float32 or tuple(s.shape) != (R, heads, D):
                raise RuntimeError("SRNL vector memories must be contiguous FP32 [directions, heads, d]")
        if len(chunk_sizes) != R:
            raise RuntimeError("Provide one chunk length per direction")
        if any(int(c) <= 0 for c in chunk_sizes):
            raise RuntimeError("Invalid SRNL chunk length or padded sequence length")
        return run_sequence((M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0), X, Q_raw, chunk_sizes,
                            q_normalized=False)


_extensions = {}


def load_fused_cuda(io_dtype=torch.bfloat16):
    if io_dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError(f"SRNL inference supports FP16, BF16, and FP32, got {io_dtype}")
    _lib.load()
    if io_dtype not in _extensions:
        _extensions[io_dtype] = _FusedModule(io_dtype)
    return _extensions[io_dtype]


@_lib.on_input_device
def srnl_sequence_inference(states, x, queries, chunk_sizes):
    """Read a packed sequence without allocating backward intermediates (fused.py:96-106)."""
    if torch.jit.is_tracing():
        raise RuntimeError("SRNL TorchScript tracing is unsupported; use eager or CUDA Graph inference")
    if torch.is_grad_enabled():
        raise RuntimeError("SRNL inference requires disabled gradients")
    memories = tuple(state.contiguous().float() for state in states)
    return load_fused_cuda(x.dtype).srnl_sequence_forward(
        *memories, x.contiguous(), queries.contiguous(), chunk_sizes)
