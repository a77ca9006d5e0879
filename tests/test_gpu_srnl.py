"""GPU parity of the SRNL kernels against the CPU oracle (double precision).

Tolerances: fp32 results within 1e-4 normwise relative error (the north-star fp32 bar);
results stored in bf16/fp16 within one rounding of the output dtype (1e-2 / 2e-3).
"""
import zlib

import numpy as np
import pytest
import torch

from tests.conftest import make_memories, rel_err, serialize_np

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(autouse=True)
def _warp_scan(monkeypatch):
    """These cases pin the warp-per-chain and CTA-lockstep scans; the chunk-parallel
    tensor-core scan, which the library picks for launches with few chains, has its own
    tests (test_gpu_tc.py)."""
    monkeypatch.setenv("VH_SRNL_SCAN", "warp")
OUT_TOL = {"f32": 1e-4, "bf16": 1e-2, "f16": 2e-3}


def _t(a, dev, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)


def _round(a, dt):
    """Round a float array through the I/O dtype (the kernel sees exactly these values)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(TORCH_DT[dt]).float().numpy()


SPATIAL_CASES = [
    # (B, H, W, heads, D, io, mem kind, per-dir skip)
    (2, 8, 8, 2, 16, "bf16", "default", False),
    (2, 7, 9, 3, 16, "bf16", "stress", False),
    (1, 9, 6, 2, 16, "f32", "stress", True),
    (3, 5, 5, 1, 16, "f16", "clamp", False),
    (2, 1, 11, 2, 16, "bf16", "stress", False),
    (2, 13, 1, 2, 16, "bf16", "stress", False),
    (1, 70, 9, 1, 16, "bf16", "stress", False),   # column chunk > one token tile
    (1, 6, 130, 1, 16, "f32", "stress", False),   # row chunk > two token tiles
    (2, 6, 6, 2, 4, "bf16", "stress", False),
    (1, 5, 7, 2, 8, "f32", "stress", True),
    (1, 6, 5, 2, 32, "bf16", "stress", False),
    (1, 4, 5, 1, 64, "f32", "stress", False),
    (5, 14, 14, 3, 16, "bf16", "stress", False),  # odd pair count per CTA
    (1, 56, 56, 2, 16, "bf16", "stress", False),  # VisionHOPE-T stage 1 (tensor-core P1, 64-token tiles)
    (2, 28, 28, 4, 16, "bf16", "clamp", True),    # stage 2 (32-token tiles)
    (1, 33, 17, 2, 16, "bf16", "stress", False),  # odd sizes: coincident middle row and column
    (1, 7, 7, 3, 16, "bf16", "stress", False),    # stage 4 (CUDA-core P1)
]


@pytest.mark.parametrize("case", SPATIAL_CASES, ids=lambda c: "x".join(map(str, c)))
@pytest.mark.parametrize("layout", ["scans", "image"])
@pytest.mark.parametrize("concurrent", [True, False], ids=["one-launch", "two-pass"])
def test_spatial_operator_matches_oracle(case, layout, concurrent, oracle, cuda):
    from visionhope_b200.srnl_core.fused import spatial_forward

    B, H, W, heads, D, io, kind, per_dir = case
    C = heads * D
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    mems = make_memories(4, heads, D, kind, gen)
    img = _round(gen.normal(size=(B, H, W, C)), io)
    qimg = _round(gen.normal(size=(B, H, W, C)), io)
    skip = gen.normal(0, 0.5, size=(4 * C,) if per_dir else (C,)).astype(np.float32)
    weights = gen.normal(1.0, 0.3, size=(4, C)).astype(np.float32)
    xs, qs = serialize_np(img), serialize_np(qimg)
    expected = oracle.srnl_spatial(mems, xs, qs, skip, weights, H, W, D)
    dev_mems = [_t(m, cuda) for m in mems]
    if layout == "scans":
        x, q = _t(xs, cuda, TORCH_DT[io]), _t(qs, cuda, TORCH_DT[io])
    else:
        x, q = _t(img, cuda, TORCH_DT[io]), _t(qimg, cuda, TORCH_DT[io])
    out = spatial_forward(dev_mems, x, q, _t(skip, cuda), _t(weights, cuda), H, W, D, layout=layout,
                          concurrent=concurrent)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and tuple(out.shape) == (B, H, W, C)
    err = rel_err(out.cpu().numpy(), expected)
    assert err < 1e-4, err


@pytest.mark.parametrize("concurrent", [True, False], ids=["one-launch", "two-pass"])
def test_spatial_is_deterministic(concurrent, oracle, cuda):
    from visionhope_b200.srnl_core.fused import spatial_forward

    gen = np.random.default_rng(7)
    B, H, W, heads, D = 3, 15, 11, 2, 16
    C = heads * D
    mems = [_t(m, cuda) for m in make_memories(4, heads, D, "stress", gen)]
    x = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    q = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    skip, wts = _t(gen.normal(size=C), cuda), _t(gen.normal(1, 0.2, size=(4, C)), cuda)
    a = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", concurrent=concurrent)
    b = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", concurrent=concurrent)
    assert torch.equal(a, b)


FINAL_CASES = [
    # (B, H, W, heads, D, io, final dtype)
    (2, 14, 14, 2, 16, "bf16", "bf16"),   # one launch: the CTA folds planes, addend and cast
    (1, 9, 17, 3, 16, "bf16", "f32"),
    (2, 7, 7, 2, 16, "bf16", "f16"),      # small image: two passes + finalize launch
    (1, 6, 5, 2, 8, "f32", "bf16"),       # CUDA-core scans + finalize launch
]


@pytest.mark.parametrize("case", FINAL_CASES, ids=lambda c: "x".join(map(str, c)))
def test_spatial_final_output_with_addend(case, oracle, cuda):
    """(final dtype)(sum of the scans + addend): equal, bit for bit, to the fp32 result plus the
    addend in fp32 and one cast (the reference's `out + lepe` then autocast's cast)."""
    from visionhope_b200.srnl_core.fused import spatial_forward

    B, H, W, heads, D, io, fdt = case
    C = heads * D
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    mems = [_t(m, cuda) for m in make_memories(4, heads, D, "stress", gen)]
    x = _t(gen.normal(size=(B, H, W, C)), cuda, TORCH_DT[io])
    q = _t(gen.normal(size=(B, H, W, C)), cuda, TORCH_DT[io])
    add = _t(gen.normal(size=(B, H, W, C)), cuda, TORCH_DT[io])
    skip, wts = _t(gen.normal(size=C), cuda), _t(gen.normal(1, 0.2, size=(4, C)), cuda)
    ref = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image")
    fin = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", addend=add,
                          final_dtype=TORCH_DT[fdt])
    assert fin.dtype == TORCH_DT[fdt] and tuple(fin.shape) == (B, H, W, C)
    assert torch.equal(fin, (ref + add.float()).to(TORCH_DT[fdt]))
    with pytest.raises(RuntimeError, match="addend requires"):
        spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", addend=add)


SEQ_CASES = [
    # (B, R, heads, L, D, chunks, x dtype, q mode, mem kind)
    (2, 1, 4, 196, 16, [14], "f32", "raw", "default"),        # config 1 shape
    (2, 1, 4, 196, 16, [14], "f32", "raw", "stress"),
    (2, 4, 3, 50, 16, [7, 7, 10, 10], "bf16", "raw", "stress"),
    (2, 4, 2, 45, 16, [9, 9, 5, 5], "f32", "norm", "stress"),
    (1, 2, 2, 100, 16, [64, 64], "bf16", "raw", "clamp"),     # tail padding
    (1, 4, 1, 300, 16, [130, 130, 75, 75], "f32", "raw", "stress"),  # long chunks
    (3, 4, 2, 20, 8, [20, 20, 20, 20], "f16", "raw", "stress"),
    (1, 1, 2, 33, 32, [16], "f32", "norm", "stress"),
    (1, 4, 1, 12, 64, [4, 4, 3, 3], "bf16", "norm", "stress"),
    (2, 2, 2, 17, 4, [5, 3], "f32", "raw", "stress"),
    (2, 4, 2, 196, 16, [14, 14, 14, 14], "bf16", "raw", "stress"),   # tensor-core P1, 16-token tiles
    (1, 2, 1, 300, 16, [100, 33], "bf16", "raw", "clamp"),          # multi-tile chunks + padding
]


@pytest.mark.parametrize("case", SEQ_CASES, ids=lambda c: "-".join(map(str, c)).replace(" ", ""))
def test_sequence_matches_oracle(case, oracle, cuda):
    from visionhope_b200.srnl_core.chunk import run_sequence

    B, R, heads, L, D, chunks, xdt, qmode, kind = case
    C = heads * D
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    mems = make_memories(R, heads, D, kind, gen)
    x = _round(gen.normal(size=(B, R, heads, L, D)), xdt)
    if qmode == "raw":
        q = _round(gen.normal(size=(B, R, L, C)), xdt)
        qt = _t(q, cuda, TORCH_DT[xdt])
    else:
        q = gen.normal(size=(B, R, heads, L, D))
        q = (q / np.linalg.norm(q, axis=-1, keepdims=True)).astype(np.float32)
        qt = _t(q, cuda)
    expected = oracle.srnl_sequence(mems, x, q, chunks, q_normalized=qmode == "norm")
    y = run_sequence([_t(m, cuda) for m in mems], _t(x, cuda, TORCH_DT[xdt]), qt, chunks,
                     q_normalized=qmode == "norm")
    torch.cuda.synchronize()
    assert y.dtype == TORCH_DT[xdt]
    err = rel_err(y.float().cpu().numpy(), expected)
    assert err < OUT_TOL[xdt], err


def test_sequence_per_chain_memories(oracle, cuda):
    from visionhope_b200.srnl_core.chunk import run_sequence

    gen = np.random.default_rng(11)
    B, R, heads, L, D = 2, 4, 2, 40, 16
    mems = make_memories(R, heads, D, "stress", gen, batch=B)
    x = gen.normal(size=(B, R, heads, L, D)).astype(np.float32)
    q = gen.normal(size=(B, R, L, heads * D)).astype(np.float32)
    expected = oracle.srnl_sequence(mems, x, q, [8, 8, 5, 5])
    y = run_sequence([_t(m, cuda) for m in mems], _t(x, cuda), _t(q, cuda), [8, 8, 5, 5],
                     q_normalized=False)
    assert rel_err(y.cpu().numpy(), expected) < 1e-4


def test_chunk_padding_equals_explicit_zero_tokens(oracle, cuda):
    """A ragged tail behaves exactly like explicit zero tokens (models/srnl_core/chunk.py:202-206)."""
    from visionhope_b200.srnl_core.chunk import run_sequence

    gen = np.random.default_rng(5)
    B, R, heads, L, D, chunk = 1, 1, 2, 23, 16, 8
    mems = [_t(m, cuda) for m in make_memories(R, heads, D, "stress", gen)]
    x = gen.normal(size=(B, R, heads, L, D)).astype(np.float32)
    q = gen.normal(size=(B, R, L, heads * D)).astype(np.float32)
    pad = 24 - L
    xp = np.concatenate([x, np.zeros((B, R, heads, pad, D), np.float32)], axis=3)
    qp = np.concatenate([q, np.zeros((B, R, pad, heads * D), np.float32)], axis=2)
    y = run_sequence(mems, _t(x, cuda), _t(q, cuda), [chunk], q_normalized=False)
    yp = run_sequence(mems, _t(xp, cuda), _t(qp, cuda), [chunk], q_normalized=False)
    assert torch.equal(y, yp[:, :, :, :L])
