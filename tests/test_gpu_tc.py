"""GPU parity of the chunk-parallel tensor-core scan (csrc/srnl_tc.cu) against the CPU oracle.

The scan is forced with VH_SRNL_SCAN=tc.  Shapes cover one and several TMA boxes per chunk
(rows and columns longer than 256 tokens), several passes per chunk (chunks longer than 512,
forward and reversed), odd and rectangular images, the serialized-scans layout of the
reference API, the final-dtype output with an addend, and packed sequences with padding and
per-direction chunk lengths.  Tolerances as elsewhere: fp32 outputs 1e-4 normwise, bf16
outputs one rounding (1e-2).  Every test also checks that no bounded wait gave up.
"""
import zlib

import numpy as np
import pytest
import torch

from tests.conftest import make_memories, rel_err, serialize_np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _force_tc(monkeypatch):
    from visionhope_b200 import _lib

    monkeypatch.setenv("VH_SRNL_SCAN", "tc")
    _lib.load().vh_tc_status(1)
    yield
    assert _lib.load().vh_tc_status(1) == 0, "a bounded wait of the tensor-core scan gave up"


def _t(a, dev, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _launches(fn):
    from visionhope_b200 import _lib

    n0 = _lib.launch_count
    out = fn()
    return out, _lib.launch_count - n0


SPATIAL = [
    # (B, H, W, heads, mem kind)
    (1, 8, 8, 1, "stress"),
    (2, 7, 9, 3, "stress"),
    (2, 14, 14, 2, "clamp"),
    (1, 56, 56, 2, "stress"),
    (1, 70, 9, 1, "stress"),
    (1, 6, 130, 1, "stress"),
    (1, 5, 300, 1, "stress"),    # rows of 300: two TMA boxes per chunk
    (1, 3, 600, 1, "stress"),    # rows of 600: two passes per chunk (reversed too)
    (1, 520, 3, 1, "clamp"),     # columns of 520: two passes per chunk
    (1, 1, 11, 2, "stress"),
    (1, 13, 1, 2, "default"),
]


@pytest.mark.parametrize("case", SPATIAL, ids=lambda c: "x".join(map(str, c)))
@pytest.mark.parametrize("layout", ["image", "scans"])
def test_tc_spatial_matches_oracle(case, layout, oracle, cuda):
    from visionhope_b200.srnl_core.fused import spatial_forward

    B, H, W, heads, kind = case
    D, C = 16, heads * 16
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    mems = make_memories(4, heads, D, kind, gen)
    img = _bf(gen.normal(size=(B, H, W, C)))
    qimg = _bf(gen.normal(size=(B, H, W, C)))
    skip = gen.normal(0, 0.5, size=C).astype(np.float32)
    weights = gen.normal(1.0, 0.3, size=(4, C)).astype(np.float32)
    xs, qs = serialize_np(img), serialize_np(qimg)
    expected = oracle.srnl_spatial(mems, xs, qs, skip, weights, H, W, D)
    src = (xs, qs) if layout == "scans" else (img, qimg)
    x, q = _t(src[0], cuda, torch.bfloat16), _t(src[1], cuda, torch.bfloat16)
    out, n = _launches(lambda: spatial_forward([_t(m, cuda) for m in mems], x, q, _t(skip, cuda),
                                               _t(weights, cuda), H, W, D, layout=layout))
    torch.cuda.synchronize()
    assert n == 2  # the scan and the fold of the four planes
    err = rel_err(out.cpu().numpy(), expected)
    assert err < 1e-4, err


def test_tc_config5_stage1_shape(oracle, cuda):
    """VisionHOPE-B stage 1 at 512 x 2048: 128 x 512 tokens, 3 heads, batch 2."""
    from visionhope_b200.srnl_core.fused import spatial_forward

    B, H, W, heads, D = 2, 128, 512, 3, 16
    C = heads * D
    gen = np.random.default_rng(4)
    mems = make_memories(4, heads, D, "stress", gen)
    img, qimg = _bf(gen.normal(size=(B, H, W, C))), _bf(gen.normal(size=(B, H, W, C)))
    skip = gen.normal(0, 0.5, size=C).astype(np.float32)
    weights = gen.normal(1.0, 0.3, size=(4, C)).astype(np.float32)
    expected = oracle.srnl_spatial(mems, serialize_np(img), serialize_np(qimg), skip, weights, H, W, D)
    out = spatial_forward([_t(m, cuda) for m in mems], _t(img, cuda, torch.bfloat16), _t(qimg, cuda, torch.bfloat16),
                          _t(skip, cuda), _t(weights, cuda), H, W, D, layout="image")
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), expected) < 1e-4


@pytest.mark.parametrize("fdt", [torch.bfloat16, torch.float32])
def test_tc_final_output_with_addend(fdt, cuda):
    """(final dtype)(sum + addend) equals the fp32 sum plus the addend, cast once."""
    from visionhope_b200.srnl_core.fused import spatial_forward

    B, H, W, heads, D = 2, 9, 17, 2, 16
    C = heads * D
    gen = np.random.default_rng(11)
    mems = [_t(m, cuda) for m in make_memories(4, heads, D, "stress", gen)]
    x = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    q = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    add = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    skip, wts = _t(gen.normal(size=C), cuda), _t(gen.normal(1, 0.2, size=(4, C)), cuda)
    ref = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image")
    fin = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", addend=add, final_dtype=fdt)
    assert fin.dtype == fdt
    assert torch.equal(fin, (ref + add.float()).to(fdt))


def test_tc_matches_warp_scan_bitwise_determinism(cuda):
    """Two runs give identical bits, and the warp-per-chain scan agrees within 1e-4."""
    import os

    from visionhope_b200.srnl_core.fused import spatial_forward

    gen = np.random.default_rng(7)
    B, H, W, heads, D = 3, 15, 11, 2, 16
    C = heads * D
    mems = [_t(m, cuda) for m in make_memories(4, heads, D, "stress", gen)]
    x = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    q = _t(gen.normal(size=(B, H, W, C)), cuda, torch.bfloat16)
    skip, wts = _t(gen.normal(size=C), cuda), _t(gen.normal(1, 0.2, size=(4, C)), cuda)
    a = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image")
    b = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image")
    os.environ["VH_SRNL_SCAN"] = "warp"
    w = spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image")
    os.environ["VH_SRNL_SCAN"] = "tc"
    assert torch.equal(a, b)
    assert rel_err(a, w) < 1e-4


SEQUENCE = [
    # (B, R, heads, L, chunks)
    (2, 1, 2, 64, [8]),
    (2, 1, 3, 47, [14]),       # padded last chunk
    (1, 2, 2, 120, [56, 7]),
    (1, 4, 1, 300, [130, 300, 40, 64]),
    (1, 1, 2, 1100, [600]),    # two passes per chunk, padded
    (2, 1, 1, 30, [64]),       # one chunk longer than the sequence
]


@pytest.mark.parametrize("case", SEQUENCE, ids=lambda c: f"B{c[0]}R{c[1]}h{c[2]}L{c[3]}")
def test_tc_sequence_matches_oracle(case, oracle, cuda):
    from visionhope_b200.srnl_core.chunk import run_sequence

    B, R, heads, L, chunks = case
    D, C = 16, heads * 16
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    mems = make_memories(R, heads, D, "stress", gen)
    x = _bf(gen.normal(size=(B, R, heads, L, D)))
    q = _bf(gen.normal(size=(B, R, L, C)))
    expected = oracle.srnl_sequence(mems, x, q, chunks)
    y = run_sequence([_t(m, cuda) for m in mems], _t(x, cuda, torch.bfloat16), _t(q, cuda, torch.bfloat16),
                     chunks, q_normalized=False)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16
    assert rel_err(y.float().cpu().numpy(), expected) < 1e-2
