"""Long chunks and rectangular row/column scans, backed by libvhope.so.

Mirror of models/srnl_core/lines.py (srnl_long_chunk, srnl_variable_lines): same names,
arguments and errors.  One kernel serves every chunk length -- chunks longer than a
shared-memory tile are processed tile by tile with the gain carried in registers -- so
there is no separate "large"/"varline" kernel family.  The autograd path uses the sequence
backward (``vh_srnl_sequence_bwd``, replacing lines.py:183-399 and 402-643): any chunk length
for head_dim 16, chunks of up to 64 tokens for the other head dims (a backward through longer
ones raises).
"""
from __future__ import annotations

import torch

from .. import _lib
from . import chunk as _base

MAX_LOGICAL_CHUNK = None
SUPPORTED_HEAD_DIMS = _base.SUPPORTED_HEAD_DIMS


@_lib.on_input_device
def _long_chunk_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, chunk_size, num_heads,
                        head_dim):
    _base._check_tracing()
    if not x.is_cuda:
        raise RuntimeError("SRNL large-line qraw CUDA kernel requires CUDA tensors.")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"SRNL large-line qraw CUDA kernel supports fp16/bf16/fp32 x, got {x.dtype}.")
    if q_raw.dtype != x.dtype:
        raise RuntimeError(
            f"SRNL large-line qraw CUDA kernel expects q_raw dtype to match x dtype, got {q_raw.dtype} vs {x.dtype}.")
    B, directions, x_num_heads, seq_len, x_head_dim = x.shape
    if directions not in (1, 2, 4) or x_num_heads != num_heads or x_head_dim != head_dim:
        raise AssertionError("Invalid x shape for large-line qraw kernel.")
    if q_raw.dim() != 4 or q_raw.shape[0] != B or q_raw.shape[1] != directions or q_raw.shape[2] != seq_len:
        raise AssertionError("Invalid q_raw shape for large-line qraw kernel.")
    if q_raw.shape[3] != num_heads * head_dim:
        raise AssertionError("q_raw channel count does not match num_heads * head_dim.")
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(f"large-line CUDA kernel requires head_dim in {SUPPORTED_HEAD_DIMS}, got {head_dim}.")
    if chunk_size <= _base.MAX_CHUNK:
        raise ValueError("large-line CUDA kernel is only intended for chunk_size > base MAX_CHUNK.")
    states = (M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0)
    return _base.run_sequence(states, x, q_raw, [chunk_size] * directions, q_normalized=False)


def srnl_long_chunk(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, chunk_size, num_heads, head_dim):
    """Recurrence with chunks longer than MAX_CHUNK (lines.py:396-399)."""
    return _base._apply(lambda: _long_chunk_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw,
                                                    int(chunk_size), int(num_heads), int(head_dim)),
                        [int(chunk_size)] * x.shape[1], False, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw)


@_lib.on_input_device
def _variable_lines_forward(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, row_chunk_size,
                            col_chunk_size, num_heads, head_dim):
    _base._check_tracing()
    if not x.is_cuda:
        raise RuntimeError("SRNL varline qraw CUDA kernel requires CUDA tensors.")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"SRNL varline qraw CUDA kernel supports fp16/bf16/fp32 x, got {x.dtype}.")
    if q_raw.dtype != x.dtype:
        raise RuntimeError(
            f"SRNL varline qraw CUDA kernel expects q_raw dtype to match x dtype, got {q_raw.dtype} vs {x.dtype}.")
    B, directions, x_num_heads, seq_len, x_head_dim = x.shape
    if directions != 4 or x_num_heads != num_heads or x_head_dim != head_dim:
        raise AssertionError("Invalid x shape for varline qraw kernel.")
    if q_raw.dim() != 4 or q_raw.shape[0] != B or q_raw.shape[1] != 4 or q_raw.shape[2] != seq_len:
        raise AssertionError("Invalid q_raw shape for varline qraw kernel.")
    if q_raw.shape[3] != num_heads * head_dim:
        raise AssertionError("q_raw channel count does not match num_heads * head_dim.")
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(f"varline CUDA kernel requires head_dim in {SUPPORTED_HEAD_DIMS}, got {head_dim}.")
    if row_chunk_size <= 0 or col_chunk_size <= 0:
        raise ValueError("row_chunk_size and col_chunk_size must be positive.")
    if seq_len % row_chunk_size != 0 or seq_len % col_chunk_size != 0:
        raise ValueError(
            f"seq_len={seq_len} must be divisible by row_chunk_size={row_chunk_size} and col_chunk_size={col_chunk_size}.")
    states = (M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0)
    chunks = [row_chunk_size, row_chunk_size, col_chunk_size, col_chunk_size]
    return _base.run_sequence(states, x, q_raw, chunks, q_normalized=False)


def srnl_variable_lines(M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, row_chunk_size,
                        col_chunk_size, num_heads, head_dim):
    """Four scans with row chunk W for directions 0-1 and column chunk H for 2-3 (lines.py:646-671)."""
    chunks = [int(row_chunk_size)] * 2 + [int(col_chunk_size)] * 2
    return _base._apply(lambda: _variable_lines_forward(
        M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw, int(row_chunk_size), int(col_chunk_size),
        int(num_heads), int(head_dim)), chunks, False, M_m_0, M_v_0, M_k_0, M_eta_0, M_alpha_0, x, q_raw)
