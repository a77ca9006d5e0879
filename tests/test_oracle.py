"""CPU tests of the oracle: pinned against the reference's own outputs (golden fixtures from
its CUDA kernels and its CPU GRN/LayerNorm code), an independent numpy restatement of the
recurrence, and composition identities between the oracle's entry points."""
import json
from pathlib import Path

import numpy as np
import pytest

from tests.conftest import make_memories, rel_err, serialize_np

GOLDEN = Path(__file__).resolve().parent / "golden"
CONSTS = (0.025, 0.0, 2.197224577, 0.999, 2 * 0.999999, 1.0)


def numpy_chain(mems, x, q, chunk, q_normalized=False):
    """Straight-line numpy restatement of one chain (inference_recurrence.cuh:4-137)."""
    Mm, Mv, Mk, e, a = (np.array(m, dtype=np.float64) for m in mems)
    L, D = x.shape
    y = np.zeros((L, D))
    step, amin, bias, mu, factor, _ = CONSTS
    for c in range((L + chunk - 1) // chunk):
        G = np.eye(D)
        for t in range(chunk):
            tt = c * chunk + t
            xv = x[tt].astype(np.float64) if tt < L else np.zeros(D)
            qv = q[tt].astype(np.float64) if tt < L else np.zeros(D)
            if not q_normalized:
                qv = qv / max(np.linalg.norm(qv), 1e-12)
            if tt < L:
                y[tt] = Mm @ qv
            kr, v = Mk @ xv, Mv @ xv
            k = kr / np.sqrt(kr @ kr + 1e-6)
            ep = np.clip(xv @ e, -10, 10)
            ap = np.clip(xv @ a + bias, -10, 10)
            eta = step * (ep if ep > 20 else np.log1p(np.exp(ep)))
            alpha = amin + (1 - amin) / (1 + np.exp(-ap))
            dn = np.sqrt((k - v) @ (k - v) + 1e-12)
            cap = mu * (1 - alpha) / (dn + 1e-6)
            eff = cap * -np.expm1(-eta / cap)
            eff = min(eff, np.nextafter(factor * alpha / max(k @ k, 1e-20), 0))
            r = (k - v) + G @ k
            G = alpha * G - eff * np.outer(r, k)
        Mm, Mv, Mk = Mm @ G, Mv @ G, Mk @ G
        e, a = G.T @ e, G.T @ a
    return y


@pytest.mark.parametrize("kind", ["default", "stress", "clamp"])
@pytest.mark.parametrize("L,chunk", [(24, 8), (23, 8), (9, 9), (5, 16)])
def test_oracle_matches_numpy_restatement(oracle, kind, L, chunk):
    gen = np.random.default_rng(L * 31 + chunk)
    D = 8
    mems = make_memories(1, 1, D, kind, gen)
    x = gen.normal(size=(1, 1, 1, L, D)).astype(np.float32)
    q = gen.normal(size=(1, 1, L, D)).astype(np.float32)
    got = oracle.srnl_sequence(mems, x, q, [chunk])[0, 0, 0]
    want = numpy_chain([m[0, 0] for m in mems], x[0, 0, 0], q[0, 0], chunk)
    assert rel_err(got, want) < 1e-12


def test_oracle_float_port_tracks_double(oracle):
    gen = np.random.default_rng(1)
    mems = make_memories(4, 2, 16, "stress", gen)
    B, H, W, C = 2, 6, 7, 32
    img, qimg = gen.normal(size=(B, H, W, C)), gen.normal(size=(B, H, W, C))
    args = (mems, serialize_np(img), serialize_np(qimg), np.zeros(C, np.float32),
            np.ones((4, C), np.float32), H, W, 16)
    assert rel_err(oracle.srnl_spatial(*args, use_f32=True), oracle.srnl_spatial(*args)) < 1e-4


@pytest.mark.parametrize("per_dir", [False, True])
def test_spatial_equals_sequence_plus_fusion(oracle, per_dir):
    """srnl_line_forward_seq == srnl_variable_lines scans followed by direction fusion."""
    gen = np.random.default_rng(2)
    B, H, W, heads, D = 2, 5, 7, 2, 16
    C, L = heads * D, H * W
    mems = make_memories(4, heads, D, "stress", gen)
    img, qimg = gen.normal(size=(B, H, W, C)), gen.normal(size=(B, H, W, C))
    xs, qs = serialize_np(img).astype(np.float32), serialize_np(qimg).astype(np.float32)
    skip = gen.normal(size=(4, heads, D) if per_dir else (heads, D)).astype(np.float32)
    wts = gen.normal(1, 0.3, size=(4, C)).astype(np.float32)
    fused = oracle.srnl_spatial(mems, xs, qs, skip, wts, H, W, D)
    xp = xs.reshape(B, 4, L, heads, D).transpose(0, 1, 3, 2, 4).copy()
    y = oracle.srnl_sequence(mems, xp, qs, [W, W, H, H]).astype(np.float32)
    out = oracle.dirfuse(y, xp, skip, wts, H, W, channels_last=False)  # [B, C, H, W]
    assert rel_err(fused, out.transpose(0, 2, 3, 1)) < 1e-6


def test_tail_padding_equals_zero_tokens(oracle):
    gen = np.random.default_rng(3)
    mems = make_memories(1, 2, 16, "stress", gen)
    x = gen.normal(size=(1, 1, 2, 21, 16)).astype(np.float32)
    q = gen.normal(size=(1, 1, 21, 32)).astype(np.float32)
    xp = np.concatenate([x, np.zeros((1, 1, 2, 3, 16), np.float32)], axis=3)
    qp = np.concatenate([q, np.zeros((1, 1, 3, 32), np.float32)], axis=2)
    a = oracle.srnl_sequence(mems, x, q, [8])
    b = oracle.srnl_sequence(mems, xp, qp, [8])[:, :, :, :21]
    assert np.array_equal(a, b)


def test_default_init_gates_are_constant(oracle):
    """With zero eta/alpha memories the gates never depend on the data (srnl.py:73-74):
    scaling x then changes outputs only through the projections, not through eta/alpha."""
    gen = np.random.default_rng(4)
    mems = make_memories(1, 1, 8, "default", gen)
    x = gen.normal(size=(1, 1, 1, 16, 8)).astype(np.float32)
    q = gen.normal(size=(1, 1, 16, 8)).astype(np.float32)
    y = oracle.srnl_sequence(mems, x, q, [4])
    assert np.isfinite(y).all() and np.abs(y).max() > 0


# ---------------------------- pins against the reference ------------------------------------
def _load(name):
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {name} not generated")
    return dict(np.load(path))


def _manifest(name="manifest.json"):
    path = GOLDEN / name
    return json.loads(path.read_text()) if path.exists() else {}


@pytest.mark.parametrize("name", sorted(k for k, v in _manifest().items() if v["kind"] == "spatial"))
def test_oracle_matches_reference_fused_kernel(oracle, name):
    meta, g = _manifest()[name], _load(name)
    mems = (g["M_m"], g["M_v"], g["M_k"], g["M_eta"], g["M_alpha"])
    got = oracle.srnl_spatial(mems, g["xs"], g["qs"], g["skip"], g["weight"], meta["H"], meta["W"], meta["D"])
    assert rel_err(got, g["out"]) < 1e-4


@pytest.mark.parametrize("name", sorted(k for k, v in _manifest().items() if v["kind"] == "sequence"))
def test_oracle_matches_reference_sequence_kernels(oracle, name):
    meta, g = _manifest()[name], _load(name)
    mems = (g["M_m"], g["M_v"], g["M_k"], g["M_eta"], g["M_alpha"])
    got = oracle.srnl_sequence(mems, g["x"], g["q"], meta["chunks"], q_normalized=meta["q_mode"] == "norm")
    bf16_out = "bfloat16" in meta["io"]
    # reference outputs stored in bf16 carry one bf16 rounding (2^-8 relative)
    assert rel_err(got, g["y"]) < (1e-2 if bf16_out else 1e-4)


@pytest.mark.parametrize("name", sorted(k for k, v in _manifest().items() if v["kind"] == "qnorm"))
def test_oracle_matches_reference_qnorm(oracle, name):
    meta, g = _manifest()[name], _load(name)
    out, inv = oracle.qnorm(g["q"], meta["heads"], meta["D"])
    assert rel_err(out, g["out"]) < 1e-6
    assert rel_err(inv, g["inv"]) < 1e-6


@pytest.mark.parametrize("name", sorted(k for k, v in _manifest().items() if v["kind"] == "dirfuse"))
def test_oracle_matches_reference_dirfuse(oracle, name):
    meta, g = _manifest()[name], _load(name)
    out = oracle.dirfuse(g["y"], g["x"], g["skip"], g["scale"], meta["H"], meta["W"], channels_last=False)
    assert rel_err(out, g["out"]) < 1e-6


@pytest.mark.parametrize("name", sorted(k for k, v in _manifest().items() if v["kind"] == "grn"))
def test_oracle_matches_reference_grn_kernel(oracle, name):
    g = _load(name)
    y = oracle.grn_nhwc(g["x_nhwc"], g["gamma"], g["beta"])
    assert rel_err(y, g["y_nhwc"]) < 1e-5


@pytest.mark.parametrize("name", sorted(_manifest("cpu_manifest.json")))
def test_oracle_matches_reference_cpu_code(oracle, name):
    g = _load(name)
    x = g["x_nchw"].transpose(0, 2, 3, 1)
    if name.startswith("cpu_grn"):
        y = oracle.grn_nhwc(x, g["gamma"], g["beta"])
    else:
        C = x.shape[-1]
        y = oracle.layernorm_rows(x.reshape(-1, C), g["weight"], g["bias"]).reshape(x.shape)
    assert rel_err(y, g["y_nchw"].transpose(0, 2, 3, 1)) < 1e-5
