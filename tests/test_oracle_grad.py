"""The gradient oracle (oracle/grad.py), pinned on the CPU: its forward restatements against the
C oracle (itself pinned against the reference's kernels and the golden fixtures), against the
golden fixtures the reference's kernels produced, and against the reference's own CPU code where
it has some (utils/grn.py:grn_reference); its gradients against finite differences."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import grad as og
from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def _rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("heads,D", [(2, 16), (3, 8), (1, 64)])
def test_qnorm_matches_c_oracle(heads, D):
    g = np.random.default_rng(heads * D)
    q = g.normal(size=(2, 4, 11, heads * D)).astype(np.float32)
    q[0, 1, 3] = 0.0  # a zero vector takes the clamped branch
    exp, _ = oracle.qnorm(q, heads, D)
    got = og.qnorm(torch.from_numpy(q).double(), heads, D).numpy()
    assert _rel(got, exp) < 1e-6


def test_qnorm_matches_golden():
    z = np.load(GOLDEN / "qnorm_bf16.npz")  # the reference's kernel on bf16 queries
    heads, D = z["out"].shape[2], z["out"].shape[4]
    got = og.qnorm(torch.from_numpy(z["q"].astype(np.float32)).double(), heads, D).numpy()
    assert _rel(got, z["out"]) < 1e-5


@pytest.mark.parametrize("per_dir", [False, True])
def test_dirfuse_matches_c_oracle(per_dir):
    g = np.random.default_rng(7 + per_dir)
    B, heads, D, H, W = 2, 3, 8, 5, 7
    C, L = heads * D, H * W
    y = g.normal(size=(B, 4, heads, L, D)).astype(np.float32)
    x = g.normal(size=(B, 4, heads, L, D)).astype(np.float32)
    skip = g.normal(size=(4, C) if per_dir else (C,)).astype(np.float32)
    scale = g.normal(size=(4, C)).astype(np.float32)
    exp = oracle.dirfuse(y, x, skip, scale, H, W, False)
    got = og.dirfuse(*(torch.from_numpy(a).double() for a in (y, x, skip, scale)), H, W).numpy()
    assert _rel(got, exp) < 1e-6


def test_layernorm_matches_c_oracle():
    g = np.random.default_rng(3)
    x = g.normal(size=(37, 96)).astype(np.float32)
    w = g.normal(size=96).astype(np.float32)
    b = g.normal(size=96).astype(np.float32)
    exp = oracle.layernorm_rows(x, w, b, 1e-6)
    got = og.layernorm_rows(*(torch.from_numpy(a).double() for a in (x, w, b)), 1e-6).numpy()
    assert _rel(got, exp) < 1e-6


def test_grn_matches_c_oracle_and_reference_fixture():
    g = np.random.default_rng(5)
    x = g.normal(size=(2, 6, 5, 24)).astype(np.float32)  # NHWC
    gamma = g.normal(size=24).astype(np.float32)
    beta = g.normal(size=24).astype(np.float32)
    exp = oracle.grn_nhwc(x, gamma, beta, 1e-6)
    xt = torch.from_numpy(x).double().permute(0, 3, 1, 2)
    got = og.grn(xt, torch.from_numpy(gamma).double(), torch.from_numpy(beta).double(), 1e-6)
    assert _rel(got.permute(0, 2, 3, 1).numpy(), exp) < 1e-6
    # The reference's own CPU GRN (utils/grn.py:26-38, eps 1e-6) produced this fixture.
    z = np.load(GOLDEN / "cpu_grn_7x7x768.npz")
    got = og.grn(torch.from_numpy(z["x_nchw"]).double(), torch.from_numpy(z["gamma"]).double().reshape(-1),
                 torch.from_numpy(z["beta"]).double().reshape(-1), 1e-6)
    assert _rel(got.numpy(), z["y_nchw"]) < 1e-5


def test_gradients_match_finite_differences():
    torch.manual_seed(0)
    q = torch.randn(1, 4, 3, 8, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda t: og.qnorm(t, 2, 4), (q,))
    y = torch.randn(1, 4, 2, 6, 4, dtype=torch.float64, requires_grad=True)
    x = torch.randn(1, 4, 2, 6, 4, dtype=torch.float64, requires_grad=True)
    sk = torch.randn(8, dtype=torch.float64, requires_grad=True)
    sc = torch.randn(4, 8, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda a, b, c, d: og.dirfuse(a, b, c, d, 2, 3), (y, x, sk, sc))
    xg = torch.randn(2, 5, 3, 4, dtype=torch.float64, requires_grad=True)
    gm = torch.randn(5, dtype=torch.float64, requires_grad=True)
    bt = torch.randn(5, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda a, b, c: og.grn(a, b, c, 1e-6), (xg, gm, bt))


@pytest.mark.parametrize("q_normalized,per_chain", [(False, False), (True, True)])
def test_srnl_sequence_matches_c_oracle(q_normalized, per_chain):
    from visionhope_b200.srnl_core.chunk import recurrence_constants_tuple

    g = np.random.default_rng(11 + per_chain)
    B, R, H, L, D = 2, 4, 2, 23, 8
    lead = (B, R, H) if per_chain else (R, H)
    mems = [g.normal(0, 0.35, lead + (D, D)).astype(np.float32) for _ in range(3)]
    mems += [g.normal(0, 0.6, lead + (D,)).astype(np.float32) for _ in range(2)]
    x = g.normal(size=(B, R, H, L, D)).astype(np.float32)
    if q_normalized:
        q = g.normal(size=(B, R, H, L, D)).astype(np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
    else:
        q = g.normal(size=(B, R, L, H * D)).astype(np.float32)
    chunks = [6, 6, 5, 9]
    exp = oracle.srnl_sequence(mems, x, q, chunks, q_normalized=q_normalized)
    got = og.srnl_sequence([torch.from_numpy(m).double() for m in mems], torch.from_numpy(x).double(),
                           torch.from_numpy(q).double(), chunks, recurrence_constants_tuple(), q_normalized)
    assert _rel(got.numpy(), exp) < 1e-12


def test_residual_matches_reference_block_fallback():
    """The residual oracle (res + branch gamma mask) against the reference's own CPU code path
    for the same add: VisionHOPEBlock._residual_add (models/block.py:90-97), which on CPU tensors
    takes `x + drop_path(gamma * branch)`.  timm is not installed, so the reference's DropPath is
    the parity harness's stand-in, the identity: the mask is all ones here (the drop-path mask
    itself is compared on the GPU, where the reference takes its fused path)."""
    import importlib

    from tests.conftest import reference

    reference("dropin")
    blk_mod = importlib.import_module("visionhope.models.block")
    torch.manual_seed(0)
    blk = blk_mod.VisionHOPEBlock(32, 16, drop_path=0.4, norm_layer="layernorm2d").train()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(6, 32, 5, 7, generator=g).double()
    br = torch.randn(6, 32, 5, 7, generator=g).double()
    gamma = torch.randn(32, 1, 1, generator=g).double()
    ref = blk._residual_add(x, br, gamma)
    exp = og.residual(x, br, gamma, torch.ones(6, dtype=torch.float64))
    assert torch.allclose(ref, exp, rtol=1e-15, atol=1e-15)
