"""SRNL recurrence for chunks of up to 64 tokens, backed by libvhope.so.

Mirror of models/srnl_core/chunk.py: same names, arguments, dtype rules and errors.  The
autograd path runs the training backward ``vh_srnl_sequence_bwd`` (chunk.py:286-359, 507-588).
Recurrence constants are read from the same environment variables (chunk.py:44-58) and
passed to the kernels at run time instead of being compiled in.
"""
from __future__ import annotations

import os

import torch

from .. import _lib

MAX_CHUNK = 64
SUPPORTED_HEAD_DIMS = (4, 8, 16, 32, 64)


def _env_float(name, default):
    raw = os.environ.get(name)
    if raw is None:
        return float(default)
    try:
        return float(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be a float, got {raw!r}") from exc


STEP_SCALE = _env_float("VISIONHOPE_STEP_SCALE", 0.025)
MIN_RETENTION = _env_float("VISIONHOPE_MIN_RETENTION", 0.0)
RETENTION_BIAS = _env_float("VISIONHOPE_RETENTION_BIAS", 2.197224577)
INJECTION_MARGIN = _env_float("VISIONHOPE_INJECTION_MARGIN", 0.999)
SPECTRAL_CLAMP = True
SPECTRAL_MARGIN = _env_float("VISIONHOPE_SPECTRAL_MARGIN", 0.999999)

if not (0.0 <= MIN_RETENTION < 1.0):
    raise ValueError(f"MIN_RETENTION must be in [0, 1), got {MIN_RETENTION}")
if not (0.0 < INJECTION_MARGIN < 1.0):
    raise ValueError(f"INJECTION_MARGIN must be in (0, 1), got {INJECTION_MARGIN}")
if not (STEP_SCALE > 0.0):
    raise ValueError(f"STEP_SCALE must be positive, got {STEP_SCALE}")
if not (0.0 < SPECTRAL_MARGIN <= 1.0):
    raise ValueError(f"SPECTRAL_MARGIN must be in (0, 1], got {SPECTRAL_MARGIN}")


def recurrence_constants():
    """The constants as the C ABI struct (vh_srnl_consts)."""
    return _lib.consts(STEP_SCALE, MIN_RETENTION, RETENTION_BIAS, INJECTION_MARGIN,
                       SPECTRAL_MARGIN, SPECTRAL_CLAMP)


def recurrence_constants_tuple():
    """(step, min retention, bias, margin, 2 x spectral margin, clamp) for oracles and tests."""
    return (STEP_SCALE, MIN_RETENTION, RETENTION_BIAS, INJECTION_MARGIN, 2.0 * SPECTRAL_MARGIN,
            1.0 if SPECTRAL_CLAMP else 0.0)


def _memories_f32(states, x):
    """fp32 contiguous memories and whether they are per chain (5-dim, chunk.py:193-200)."""
    B, directions, heads, _, D = x.shape
    dims = states[0].dim()
    if dims not in (4, 5):
        raise AssertionError(
            f"Expected memory tensors with 4 or 5 dims, got shape {tuple(states[0].shape)}.")
    count = directions * heads if dims == 4 else B * directions * heads
    out = []
    for i, s in enumerate(states):
        s = s.detach().contiguous().to(device=x.device, dtype=torch.float32)
        want = count * D * D if i < 3 else count * D
        if s.numel() != want:
            raise AssertionError(f"SRNL memory {i} has {s.numel()} values, expected {want}")
        out.append(s)
    return tuple(out), dims == 5


def run_sequence(states, x, q, chunk_sizes, *, q_normalized):
    """Launch the packed recurrence: x [B,R,h,L,D]; q raw [B,R,L,C] or unit-norm fp32 [B,R,h,L,D]."""
    _lib.ensure_device(x)
    B, R, heads, L, D = x.shape
    if D not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(f"SRNL CUDA kernel requires head_dim in {SUPPORTED_HEAD_DIMS}, got {D}.")
    mems, per_chain = _memories_f32(states, x)
    x_c = x.contiguous()
    q_c = q.contiguous()
    y = torch.empty_like(x_c)
    chunks = list(int(c) for c in chunk_sizes) + [1] * (4 - len(chunk_sizes))
    args = _lib.VhSequenceArgs(
        _lib.memories(mems, per_chain), x_c.data_ptr(), q_c.data_ptr(), y.data_ptr(),
        _lib.dtype_code(x_c.dtype), _lib.dtype_code(q_c.dtype), 1 if q_normalized else 0,
        B, R, heads, L, D, (_lib.c_int32 * 4)(*chunks), recurrence_constants())
    _lib.check(_lib.load().vh_srnl_sequence_fwd(args, _lib.stream_handle(x.device)),
               "vh_srnl_sequence_fwd")
    return y


def sequence_backward(states, x, q, chunk_sizes, grad_y, *, q_normalized):
    """Gradients of :func:`run_sequence` (``vh_srnl_sequence_bwd``, replaces
    models/srnl_core/csrc/chunk.cu:511-1057): returns (dM_m, dM_v, dM_k, dM_eta, dM_alpha) in the
    memories' shapes, dx in x's shape and dq in q's shape, all fp32.  head_dim 4, 8, 16 or 32;
    any chunk length for head_dim 16, up to 64 tokens for the others."""
    _lib.ensure_device(x)
    B, R, heads, L, D = x.shape
    mems, per_chain = _memories_f32(states, x)
    x_c, q_c = x.contiguous(), q.contiguous()
    g = grad_y.contiguous().float()
    dx = torch.empty(x_c.shape, device=x.device, dtype=torch.float32)
    dq = torch.empty(q_c.shape, device=x.device, dtype=torch.float32)
    dm = [torch.empty_like(m) for m in mems]
    chunks = list(int(c) for c in chunk_sizes) + [1] * (4 - len(chunk_sizes))
    args = _lib.VhSequenceBwdArgs(
        _lib.memories(mems, per_chain), x_c.data_ptr(), q_c.data_ptr(), _lib.dtype_code(x_c.dtype),
        _lib.dtype_code(q_c.dtype), 1 if q_normalized else 0, g.data_ptr(), dx.data_ptr(), dq.data_ptr(),
        *(t.data_ptr() for t in dm), B, R, heads, L, D, (_lib.c_int32 * 4)(*chunks), recurrence_constants())
    lib = _lib.load()
    nbytes = int(lib.vh_srnl_sequence_bwd_workspace_bytes(args))
    ws = torch.empty((max(nbytes, 16) + 3) // 4, device=x.device, dtype=torch.float32)
    _lib.check(lib.vh_srnl_sequence_bwd(args, ws.data_ptr(), ws.numel() * 4, _lib.stream_handle(x.device)),
               "vh_srnl_sequence_bwd")
    return tuple(m.view(s.shape) for m, s in zip(dm, states)), dx, dq


class _SequenceFunction(torch.autograd.Function):
    """The packed recurrence with its backward (chunk.py:172-359, 366-588): the forward saves
    only its inputs; the backward recomputes the chunk states and the gain sequence."""

    @staticmethod
    def forward(ctx, forward, chunks, q_normalized, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q):
        ctx.save_for_backward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q)
        ctx.cfg = (list(chunks), bool(q_normalized))
        return forward()

    @staticmethod
    def backward(ctx, dy):
        *states, x, q = ctx.saved_tensors
        chunks, q_normalized = ctx.cfg
        dms, dx, dq = sequence_backward(states, x, q, chunks, dy, q_normalized=q_normalized)
        return (None, None, None, *(d.to(s.dtype) for d, s in zip(dms, states)), dx.to(x.dtype), dq.to(q.dtype))


def _apply(fn, chunks, q_normalized, *tensors):
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors):
        return _SequenceFunction.apply(fn, chunks, q_normalized, *tensors)
    return fn()


def _check_tracing():
    if torch.jit.is_tracing():
        raise RuntimeError("SRNL TorchScript tracing is unsupported; use eager or CUDA Graph inference.")


@_lib.on_input_device
def _normalized_query_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q, chunk_size):
    _check_tracing()
    if not x.is_cuda:
        raise RuntimeError("SRNL CUDA kernel requires CUDA tensors.")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"SRNL CUDA kernel supports fp16/bf16/fp32 x, got {x.dtype}.")
    if q.dtype != torch.float32:
        raise RuntimeError(f"SRNL normalized q path expects fp32 q, got {q.dtype}.")
    B, directions, num_heads, seq_len, head_dim = x.shape
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(
            f"SRNL CUDA kernel requires head_dim in {SUPPORTED_HEAD_DIMS}, got {head_dim}.")
    if chunk_size > MAX_CHUNK:
        raise ValueError(f"chunk_size={chunk_size} exceeds MAX_CHUNK={MAX_CHUNK} in CUDA kernel")
    if tuple(q.shape) != tuple(x.shape):
        raise AssertionError("SRNL normalized queries must have the packed input shape")
    states = (M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0)
    return run_sequence(states, x, q, [int(chunk_size)] * directions, q_normalized=True)


def srnl_normalized_query(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q, chunk_size):
    """Packed recurrence with unit-norm fp32 queries (chunk.py:628-631); y has x's dtype."""
    if x.dtype in (torch.float16, torch.bfloat16, torch.float32) and q.dtype == torch.float32:
        return _apply(lambda: _normalized_query_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0,
                                                        x, q, int(chunk_size)),
                      [int(chunk_size)] * x.shape[1], True, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q)
    raise RuntimeError("The release HOPE CUDA path expects fp16/bf16/fp32 x and fp32 normalized q.")


srnl_normalized_query.supports_broadcast_state = True


@_lib.on_input_device
def _raw_query_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, chunk_size, num_heads,
                       head_dim):
    _check_tracing()
    if not x.is_cuda:
        raise RuntimeError("SRNL qraw CUDA kernel requires CUDA tensors.")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"SRNL qraw CUDA kernel supports fp16/bf16/fp32 x, got {x.dtype}.")
    if q_raw.dtype != x.dtype:
        raise RuntimeError(
            f"SRNL qraw CUDA kernel expects q_raw dtype to match x dtype, got {q_raw.dtype} vs {x.dtype}.")
    B, directions, x_num_heads, seq_len, x_head_dim = x.shape
    if directions != 4 or x_num_heads != num_heads or x_head_dim != head_dim:
        raise AssertionError("Invalid x shape for SRNL qraw kernel.")
    if q_raw.dim() != 4 or q_raw.shape[0] != B or q_raw.shape[1] != 4 or q_raw.shape[2] != seq_len:
        raise AssertionError("Invalid q_raw shape for SRNL qraw kernel.")
    if q_raw.shape[3] != num_heads * head_dim:
        raise AssertionError("q_raw channel count does not match num_heads * head_dim.")
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(
            f"SRNL CUDA kernel requires head_dim in {SUPPORTED_HEAD_DIMS}, got {head_dim}.")
    if chunk_size > MAX_CHUNK:
        raise ValueError(f"chunk_size={chunk_size} exceeds MAX_CHUNK={MAX_CHUNK} in CUDA kernel")
    states = (M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0)
    return run_sequence(states, x, q_raw, [int(chunk_size)] * 4, q_normalized=False)


def srnl_raw_query(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, chunk_size, num_heads, head_dim):
    """Four-direction recurrence with raw queries normalized in-kernel (chunk.py:622-625)."""
    return _apply(lambda: _raw_query_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw,
                                             int(chunk_size), int(num_heads), int(head_dim)),
                  [int(chunk_size)] * 4, False, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw)


def can_fuse_raw_query(x, q_raw, num_heads, head_dim):
    if not (x.is_cuda and q_raw.is_cuda):
        return False
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32) or q_raw.dtype != x.dtype:
        return False
    if x.dim() != 5 or q_raw.dim() != 4:
        return False
    if x.shape[1] != 4 or q_raw.shape[1] != 4:
        return False
    if int(head_dim) not in SUPPORTED_HEAD_DIMS:
        return False
    return (
        int(x.shape[0]) == int(q_raw.shape[0])
        and int(x.shape[3]) == int(q_raw.shape[2])
        and int(x.shape[2]) == int(num_heads)
        and int(x.shape[4]) == int(head_dim)
        and int(q_raw.shape[3]) == int(num_heads) * int(head_dim)
    )
