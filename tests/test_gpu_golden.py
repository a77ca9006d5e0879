"""Our kernels against the reference's own kernels' outputs (tests/golden, produced on a B200
by tests/golden/make_golden.py from oracle/_ref).  fp32 outputs: 1e-4 normwise relative error;
outputs the reference stores in bf16: 1e-2 (one bf16 rounding on either side)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text()) if (GOLDEN / "manifest.json").exists() else {}
DT = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}


def _g(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def _t(a, dev, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_against_reference_kernels(name, cuda):
    meta, g = MANIFEST[name], _g(name)
    kind = meta["kind"]
    io = DT.get(meta.get("io"), torch.float32)
    if kind in ("spatial", "sequence"):
        mems = [_t(g[k], cuda) for k in ("M_m", "M_v", "M_k", "M_eta", "M_alpha")]
    if kind == "spatial":
        from visionhope_b200.srnl_core.fused import load_fused_cuda

        out = load_fused_cuda(io).srnl_line_forward_seq_noatomic(
            *mems, _t(g["xs"], cuda, io), _t(g["qs"], cuda, io), _t(g["skip"], cuda),
            _t(g["weight"], cuda), meta["H"], meta["W"], meta["D"])
        assert rel_err(out.cpu().numpy(), g["out"]) < 1e-4
    elif kind == "sequence":
        from visionhope_b200.srnl_core.chunk import run_sequence

        norm = meta["q_mode"] == "norm"
        q = _t(g["q"], cuda) if norm else _t(g["q"], cuda, io)
        y = run_sequence(mems, _t(g["x"], cuda, io), q, meta["chunks"], q_normalized=norm)
        tol = 1e-2 if io != torch.float32 else 1e-4
        assert rel_err(y.float().cpu().numpy(), g["y"]) < tol
    elif kind == "qnorm":
        from visionhope_b200.utils.query_normalization import visionhope_qnorm

        out = visionhope_qnorm(_t(g["q"], cuda, io), meta["heads"], meta["D"])
        assert rel_err(out.cpu().numpy(), g["out"]) < 1e-6
    elif kind == "dirfuse":
        from visionhope_b200.utils.direction_fusion import visionhope_postprocess_scale

        out = visionhope_postprocess_scale(_t(g["y"], cuda, io), _t(g["x"], cuda, io), _t(g["skip"], cuda),
                                           _t(g["scale"], cuda), meta["H"], meta["W"], meta["channels_last"])
        assert rel_err(out.cpu().numpy(), g["out"]) < 1e-6
    elif kind == "grn":
        from visionhope_b200.utils.grn import global_response_norm

        x = _t(g["x_nhwc"], cuda, io).permute(0, 3, 1, 2)
        y = global_response_norm(x, _t(g["gamma"], cuda), _t(g["beta"], cuda))
        assert rel_err(y.permute(0, 2, 3, 1).cpu().numpy(), g["y_nhwc"]) < 1e-5
    else:
        pytest.fail(f"unknown golden kind {kind}")
