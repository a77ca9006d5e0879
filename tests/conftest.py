"""Shared fixtures.  `-m gpu` tests need a CUDA device; everything else runs on CPU."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o


def reference(mode):
    """The reference's own modules (``oracle/refmodel.py``): "native" on the reference's own
    kernels, "dropin" over this repository's modules.  Skips when they were not staged (no
    reference checkout when ``__graft_entry__.build()`` ran)."""
    from oracle import refmodel

    if not refmodel.available():
        pytest.skip("reference package not staged (oracle/build_ref.py stage_python)")
    if mode == "native" and not refmodel.kernels_available():
        pytest.skip("reference kernels not built (oracle/build_ref.py)")
    return refmodel.load(mode)


@pytest.fixture
def ref_dropin():
    return reference("dropin")


@pytest.fixture
def ref_native():
    return reference("native")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda:0")


def _np(a):
    try:
        import torch

        if isinstance(a, torch.Tensor):
            return a.detach().float().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return a


def rel_err(actual, expected) -> float:
    """Normwise relative error max|a - e| / max|e| (0 when both are zero)."""
    a = np.asarray(_np(actual), dtype=np.float64)
    e = np.asarray(_np(expected), dtype=np.float64)
    scale = float(np.max(np.abs(e))) if e.size else 0.0
    diff = float(np.max(np.abs(a - e))) if e.size else 0.0
    return diff / scale if scale > 0 else diff


def make_memories(dirs, heads, D, kind, gen, *, batch=None):
    """SRNL initial memories as numpy fp32 (m, v, k, eta, alpha).

    kind "default": the reference init (trunc-normal std 0.01 matrices, zero vectors,
    models/srnl.py:70-74) -- the gates are then constant, so also:
    kind "stress": larger matrices and random eta/alpha memories (data-dependent gates);
    kind "clamp": retention memories pushed negative so the spectral clamp binds.
    """
    lead = (dirs, heads) if batch is None else (batch, dirs, heads)
    if kind == "default":
        mats = [np.clip(gen.normal(0, 0.01, lead + (D, D)), -0.02, 0.02) for _ in range(3)]
        vecs = [np.zeros(lead + (D,)) for _ in range(2)]
    elif kind == "stress":
        mats = [gen.normal(0, 0.35, lead + (D, D)) for _ in range(3)]
        vecs = [gen.normal(0, 0.6, lead + (D,)), gen.normal(0, 0.6, lead + (D,))]
    elif kind == "clamp":
        mats = [gen.normal(0, 0.35, lead + (D, D)) for _ in range(3)]
        vecs = [gen.normal(0.5, 1.5, lead + (D,)), gen.normal(-3.0, 1.0, lead + (D,))]
    else:
        raise ValueError(kind)
    return tuple(np.ascontiguousarray(a, dtype=np.float32) for a in (*mats, *vecs))


def serialize_np(img):
    """[B, H, W, C] image -> the four scans [B, 4, L, C] (models/operator.py:79-86)."""
    B, H, W, C = img.shape
    hw = img.reshape(B, H * W, C)
    wh = img.transpose(0, 2, 1, 3).reshape(B, H * W, C)
    return np.ascontiguousarray(np.stack([hw, hw[:, ::-1], wh, wh[:, ::-1]], axis=1))
