"""ctypes front end of the CPU oracle (``oracle/vhope_oracle.c``).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` import this module, as the checker or as the timed CPU
stand-in for the reference (which has no CPU SRNL path).  The product never does.

Every function takes numpy arrays (any float dtype; bf16 torch tensors are widened
exactly by :func:`to_f32`) and returns float64 numpy arrays.  ``use_f32`` switches
the SRNL recurrence to float arithmetic (the timed port); the default is double.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD_DIR = HERE / "_build"
LIB_PATH = BUILD_DIR / "libvhope_oracle.so"
SOURCES = [HERE / "vhope_oracle.c", HERE / "srnl_core.inc"]

# Reference recurrence constants (models/srnl_core/chunk.py:44-49): step scale,
# minimum retention, retention bias, injection margin, 2 x spectral margin, clamp on/off.
DEFAULT_CONSTS = (0.025, 0.0, 2.197224577, 0.999, 2.0 * 0.999999, 1.0)

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc/OpenMP into ``oracle/_build/`` (idempotent)."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    newest = max(p.stat().st_mtime for p in SOURCES)
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= newest:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-fno-fast-math",
           str(HERE / "vhope_oracle.c"), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        for name in ("orc_srnl_spatial", "orc_srnl_sequence", "orc_qnorm", "orc_dirfuse",
                     "orc_grn", "orc_layernorm"):
            getattr(_lib, name).restype = ctypes.c_int
    return _lib


def to_f32(a) -> np.ndarray:
    """Contiguous float32 numpy copy of a numpy array or (CPU/GPU, any float dtype) tensor."""
    try:
        import torch

        if isinstance(a, torch.Tensor):
            a = a.detach().to("cpu", torch.float32).contiguous().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _consts(consts):
    return np.ascontiguousarray(np.asarray(consts if consts is not None else DEFAULT_CONSTS,
                                           dtype=np.float64))


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


def srnl_spatial(memories, xs, q_raw, d_skip, weights, height, width, head_dim, *,
                 consts=None, use_f32=False):
    """Oracle of ``srnl_line_forward_seq_noatomic``: xs, q_raw [B,4,L,C] -> fp64 [B,H,W,C]."""
    Mm, Mv, Mk, Me, Ma = (to_f32(m) for m in memories)
    X, Q, skip, wt = to_f32(xs), to_f32(q_raw), to_f32(d_skip).reshape(-1), to_f32(weights)
    B, R, L, C = X.shape
    D = int(head_dim)
    heads = C // D
    assert R == 4 and L == height * width and heads * D == C
    out = np.empty((B, height, width, C), dtype=np.float64)
    k = _consts(consts)
    rc = lib().orc_srnl_spatial(B, int(height), int(width), heads, D, _p(Mm), _p(Mv), _p(Mk),
                                _p(Me), _p(Ma), _p(X), _p(Q), _p(skip),
                                int(skip.size == 4 * C), _p(wt), _p(k), _p(out), int(use_f32))
    _check(rc, "spatial")
    return out


def srnl_sequence(memories, x, q, chunk_sizes, *, q_normalized=False, consts=None,
                  use_f32=False):
    """Oracle of the packed recurrence: x [B,R,h,L,D]; q raw [B,R,L,C] or normalized [B,R,h,L,D].

    Memories are [R,h,D,D]/[R,h,D], or 5-dim [B,R,h,D,D]/[B,R,h,D] for one state per chain
    (models/srnl_core/chunk.py:193-200).  Returns fp64 [B,R,h,L,D].
    """
    per_chain = int(to_f32(memories[0]).ndim == 5)
    Mm, Mv, Mk, Me, Ma = (to_f32(m) for m in memories)
    X, Q = to_f32(x), to_f32(q)
    B, R, heads, L, D = X.shape
    chunks = np.ascontiguousarray(np.asarray(list(chunk_sizes), dtype=np.int32))
    assert chunks.size == R
    Y = np.empty(X.shape, dtype=np.float64)
    k = _consts(consts)
    rc = lib().orc_srnl_sequence(B, R, heads, L, D, _p(Mm), _p(Mv), _p(Mk), _p(Me), _p(Ma), _p(X),
                                 _p(Q), int(bool(q_normalized)), _p(chunks), per_chain, _p(k),
                                 _p(Y), int(use_f32))
    _check(rc, "sequence")
    return Y


def qnorm(q_raw, num_heads, head_dim):
    """Oracle of ``visionhope_qnorm``: [B,R,L,C] -> ([B,R,h,L,D], inv [B*R*L*h])."""
    Q = to_f32(q_raw)
    B, R, L, C = Q.shape
    out = np.empty((B, R, num_heads, L, head_dim), dtype=np.float64)
    inv = np.empty((B * R * L * num_heads,), dtype=np.float64)
    _check(lib().orc_qnorm(B, R, L, int(num_heads), int(head_dim), _p(Q), _p(out), _p(inv)),
           "qnorm")
    return out, inv


def dirfuse(y, x, d_skip, scale, height, width, channels_last):
    """Oracle of ``visionhope_postprocess_scale``: [B,4,h,L,D] pair -> fp64 logical [B,C,H,W]."""
    Y, X, skip, sc = to_f32(y), to_f32(x), to_f32(d_skip).reshape(-1), to_f32(scale)
    B, R, heads, L, D = Y.shape
    C = heads * D
    out = np.empty((B, C, height, width) if not channels_last else (B, height, width, C),
                   dtype=np.float64)
    _check(lib().orc_dirfuse(B, heads, int(height), int(width), D, _p(Y), _p(X), _p(skip),
                             int(skip.size == 4 * C), _p(sc), int(bool(channels_last)), _p(out)),
           "dirfuse")
    return out if not channels_last else out.transpose(0, 3, 1, 2)


def grn_nhwc(x_nhwc, gamma, beta, eps=1e-6):
    """Oracle of GRN on a physical [B,H,W,C] array -> fp64 [B,H,W,C]."""
    X, g, b = to_f32(x_nhwc), to_f32(gamma).reshape(-1), to_f32(beta).reshape(-1)
    B, H, W, C = X.shape
    Y = np.empty(X.shape, dtype=np.float64)
    _check(lib().orc_grn(B, ctypes.c_long(H * W), C, _p(X), _p(g), _p(b), ctypes.c_double(eps),
                         _p(Y)), "grn")
    return Y


def layernorm_rows(x_rows, weight, bias, eps=1e-6):
    """Oracle of a channels-last row LayerNorm: [rows, C] -> fp64 [rows, C]."""
    X, w, b = to_f32(x_rows), to_f32(weight).reshape(-1), to_f32(bias).reshape(-1)
    rows, C = X.shape
    Y = np.empty(X.shape, dtype=np.float64)
    _check(lib().orc_layernorm(ctypes.c_long(rows), C, _p(X), _p(w), _p(b), ctypes.c_double(eps),
                               _p(Y)), "layernorm")
    return Y
