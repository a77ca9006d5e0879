"""Backward kernels (vh_qnorm_bwd, vh_dirfuse_bwd, vh_layernorm_bwd, vh_grn_bwd,
vh_srnl_sequence_bwd) through the autograd Functions of the drop-in modules, against fp64 CPU
autograd of the gradient oracle (oracle/grad.py) on the same inputs.  Bar: normwise relative
error 1e-5 for fp32 gradients of the one-pass operators, 2e-4 through the SRNL recurrence (an fp32
recurrence of up to 70 tokens against fp64), one 16-bit rounding (8e-3, 1e-2 through the
recurrence) where the gradient is returned in bf16/fp16 as the reference does."""
import pytest
import torch

from oracle import grad as og

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _tol(dtype):
    return 1e-5 if dtype == torch.float32 else 8e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("heads,D,L", [(2, 16, 49), (3, 8, 20), (1, 64, 7), (6, 4, 33)])
def test_qnorm_backward(dtype, heads, D, L):
    from visionhope_b200.utils.query_normalization import visionhope_qnorm

    g = torch.Generator().manual_seed(heads * 100 + D + L)
    q = torch.randn(2, 4, L, heads * D, generator=g).to(dtype)
    if dtype != torch.float16:  # its gradient, g * 1e12, is beyond fp16's range
        q[1, 2, 3, :D] = 0  # a zero vector: the clamped branch
    gout = torch.randn(2, 4, heads, L, D, generator=g)
    qd = q.to(DEV).requires_grad_(True)
    out = visionhope_qnorm(qd, heads, D)
    out.backward(gout.to(DEV))
    (exp,) = og.grads(lambda t: og.qnorm(t, heads, D), [q.float()], gout)
    assert qd.grad.dtype == dtype and qd.grad.shape == q.shape
    assert _rel(qd.grad, exp) < _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("channels_last", [False, True])
@pytest.mark.parametrize("per_dir", [False, True])
@pytest.mark.parametrize("B,heads,D,H,W", [(2, 2, 16, 7, 9), (1, 3, 8, 14, 14), (2, 1, 32, 5, 70)])
def test_dirfuse_backward(dtype, channels_last, per_dir, B, heads, D, H, W):
    from visionhope_b200.utils.direction_fusion import visionhope_postprocess_scale

    g = torch.Generator().manual_seed(B * 1000 + heads * 100 + H + W + 7 * per_dir)
    L, C = H * W, heads * D
    y = torch.randn(B, 4, heads, L, D, generator=g).to(dtype)
    x = torch.randn(B, 4, heads, L, D, generator=g).to(dtype)
    skip = torch.randn((4, C) if per_dir else (C,), generator=g)
    scale = torch.randn(4, C, generator=g)
    gout = torch.randn(B, C, H, W, generator=g)
    leaves = [t.to(DEV).requires_grad_(True) for t in (y, x, skip, scale)]
    out = visionhope_postprocess_scale(*leaves, H, W, channels_last)
    gd = gout.to(DEV)
    if channels_last:
        gd = gd.contiguous(memory_format=torch.channels_last)
    out.backward(gd)
    exp = og.grads(lambda a, b, c, d: og.dirfuse(a, b, c, d, H, W), [y.float(), x.float(), skip, scale], gout)
    for leaf, e in zip(leaves, exp):
        assert leaf.grad.shape == e.shape
        tol = _tol(dtype) if leaf.dtype != torch.float32 else 2e-5
        assert _rel(leaf.grad, e) < tol


def test_dirfuse_backward_is_deterministic():
    from visionhope_b200.utils.direction_fusion import postprocess_backward

    g = torch.Generator().manual_seed(5)
    B, heads, D, H, W = 4, 3, 16, 28, 28
    y, x = (torch.randn(B, 4, heads, H * W, D, generator=g).to(DEV) for _ in range(2))
    skip, scale = torch.randn(heads * D, generator=g).to(DEV), torch.randn(4, heads * D, generator=g).to(DEV)
    gout = torch.randn(B, heads * D, H, W, generator=g).to(DEV)
    r1 = postprocess_backward(gout, y, x, skip, scale, H, W)
    r2 = postprocess_backward(gout, y, x, skip, scale, H, W)
    assert all(torch.equal(a, b) for a, b in zip(r1, r2))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,C,H,W", [(2, 96, 14, 14), (3, 40, 5, 7), (2, 256, 9, 9), (1, 500, 7, 7),
                                     (1, 768, 7, 7), (2, 1000, 3, 3)])
def test_layernorm_backward(dtype, B, C, H, W):
    """One-pass kernels for C <= 128 (eight lanes per row) and C <= 512 (a warp per row), the
    two-kernel path above; 500 leaves lanes without a channel."""
    from visionhope_b200.utils.layer_norm_cuda import visionhope_layernorm2d

    g = torch.Generator().manual_seed(B + C + H)
    x = (torch.randn(B, C, H, W, generator=g) * 2 + 0.5).to(dtype).contiguous(memory_format=torch.channels_last)
    w = torch.randn(C, generator=g)
    b = torch.randn(C, generator=g)
    gout = torch.randn(B, C, H, W, generator=g)
    leaves = [x.to(DEV).requires_grad_(True), w.to(DEV).requires_grad_(True), b.to(DEV).requires_grad_(True)]
    y = visionhope_layernorm2d(*leaves, 1e-6)
    y.backward(gout.to(DEV))

    def ln2d(a, ww, bb):
        return og.layernorm_rows(a.permute(0, 2, 3, 1), ww, bb, 1e-6).permute(0, 3, 1, 2)

    exp = og.grads(ln2d, [x.float(), w, b], gout)
    assert leaves[0].grad.dtype == dtype and leaves[0].grad.is_contiguous(memory_format=torch.channels_last)
    assert _rel(leaves[0].grad, exp[0]) < _tol(dtype)
    assert _rel(leaves[1].grad, exp[1]) < 2e-5
    assert _rel(leaves[2].grad, exp[2]) < 2e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,C,H,W", [(2, 96, 14, 14), (4, 64, 7, 7), (1, 2560, 4, 4), (3, 20, 9, 5)])
def test_grn_backward(dtype, B, C, H, W):
    from visionhope_b200.utils.grn_cuda import visionhope_grn

    g = torch.Generator().manual_seed(B * 7 + C + H)
    x = torch.randn(B, C, H, W, generator=g)
    x[0, 1] = 0  # a channel with Gx = 0
    x = x.to(dtype).contiguous(memory_format=torch.channels_last)
    gamma = torch.randn(C, generator=g) * 0.5
    beta = torch.randn(C, generator=g) * 0.5
    gout = torch.randn(B, C, H, W, generator=g)
    leaves = [x.to(DEV).requires_grad_(True), gamma.to(DEV).requires_grad_(True), beta.to(DEV).requires_grad_(True)]
    y = visionhope_grn(*leaves, 1e-6)
    y.backward(gout.to(DEV))
    exp = og.grads(lambda a, b, c: og.grn(a, b, c, 1e-6), [x.float(), gamma, beta], gout)
    # Where Gx = 0 the fp64 autograd of sqrt gives nan; the reference's kernel (grn_cuda.cu:
    # 256-258) takes 1/Gx as 0 there, and so do we: compare the channels with Gx > 0.
    dx = leaves[0].grad.double().cpu()
    ok = torch.isfinite(exp[0])
    assert torch.isfinite(dx).all()
    assert _rel(dx[ok], exp[0][ok]) < _tol(dtype)
    assert _rel(leaves[1].grad, exp[1].nan_to_num()) < 2e-5
    assert _rel(leaves[2].grad, exp[2]) < 2e-5


def _srnl_case(seed, B, R, H, L, D, per_chain, q_normalized, dtype, mem_scale=0.35):
    g = torch.Generator().manual_seed(seed)
    lead = (B, R, H) if per_chain else (R, H)
    mems = [torch.randn(*lead, D, D, generator=g) * mem_scale for _ in range(3)]
    mems += [torch.randn(*lead, D, generator=g) * 0.6 for _ in range(2)]
    x = torch.randn(B, R, H, L, D, generator=g).to(dtype)
    if q_normalized:
        q = torch.randn(B, R, H, L, D, generator=g)
        q = q / q.norm(dim=-1, keepdim=True)
    else:
        q = torch.randn(B, R, L, H * D, generator=g).to(dtype)
    gy = torch.randn(B, R, H, L, D, generator=g)
    return mems, x, q, gy


@pytest.mark.parametrize("q_normalized", [False, True])
@pytest.mark.parametrize("per_chain", [False, True])
@pytest.mark.parametrize("D,chunk,L,dtype,mem_scale", [
    (16, 14, 30, torch.float32, 0.35), (8, 7, 20, torch.float32, 0.35), (16, 64, 70, torch.float32, 0.35),
    (32, 5, 12, torch.float32, 0.35), (4, 9, 9, torch.float32, 0.35), (16, 12, 26, torch.float32, 1.0),
    (16, 14, 28, torch.bfloat16, 0.35), (16, 100, 230, torch.float32, 0.35), (16, 45, 100, torch.bfloat16, 1.0),
    (16, 33, 33, torch.float32, 0.35)])
def test_srnl_sequence_backward(q_normalized, per_chain, D, chunk, L, dtype, mem_scale):
    """The reference's training path (chunk.py SRNLNormalizedQueryFunction / SRNLRawQueryFunction)
    through the drop-in functions: every input's gradient against fp64 autograd of the oracle
    recurrence.  mem_scale 1.0 makes the spectral clamp bind on part of the tokens.  Chunks of
    100 and 45 tokens (head_dim 16) span several 32-token tiles of the warp backward; 33 leaves
    one token in the second tile."""
    from visionhope_b200.srnl_core.chunk import (recurrence_constants_tuple, srnl_normalized_query,
                                                  srnl_raw_query)

    B, R, H = 2, 4, 2
    mems, x, q, gy = _srnl_case(D * 100 + chunk + L, B, R, H, L, D, per_chain, q_normalized, dtype, mem_scale)
    leaves = [t.to(DEV).requires_grad_(True) for t in (*mems, x, q)]
    if chunk > 64:  # past MAX_CHUNK: srnl_long_chunk (lines.py), or the packed function itself
        from visionhope_b200.srnl_core import chunk as core
        from visionhope_b200.srnl_core.lines import srnl_long_chunk
        if q_normalized:
            y = core._apply(lambda: core.run_sequence(leaves[:5], leaves[5], leaves[6], [chunk] * R,
                                                      q_normalized=True), [chunk] * R, True, *leaves)
        else:
            y = srnl_long_chunk(*leaves, chunk, H, D)
    elif q_normalized:
        y = srnl_normalized_query(*leaves, chunk)
    else:
        y = srnl_raw_query(*leaves, chunk, H, D)
    y.backward(gy.to(DEV).to(y.dtype))

    def fn(*t):
        return og.srnl_sequence(t[:5], t[5], t[6], [chunk] * R, recurrence_constants_tuple(), q_normalized)

    exp = og.grads(fn, [*mems, x.float(), q.float()], gy.to(dtype).float())
    names = ["M_m", "M_v", "M_k", "M_eta", "M_alpha", "x", "q"]
    for name, leaf, e in zip(names, leaves, exp):
        assert leaf.grad is not None and leaf.grad.shape == leaf.shape, name
        if e is None:  # no path from this input to y (a one-chunk sequence never refreshes the state)
            assert not leaf.grad.any(), name
            continue
        tol = 2e-4 if leaf.grad.dtype == torch.float32 else 1e-2
        err = _rel(leaf.grad, e)
        assert err < tol, f"{name}: {err:.3e}"


def test_srnl_sequence_backward_is_deterministic():
    from visionhope_b200.srnl_core.chunk import recurrence_constants, sequence_backward

    mems, x, q, gy = _srnl_case(3, 3, 4, 2, 40, 16, False, False, torch.float32)
    args = ([m.to(DEV) for m in mems], x.to(DEV), q.to(DEV), [14] * 4, gy.to(DEV))
    r1 = sequence_backward(*args, q_normalized=False)
    r2 = sequence_backward(*args, q_normalized=False)
    flat1 = [*r1[0], r1[1], r1[2]]
    flat2 = [*r2[0], r2[1], r2[2]]
    assert all(torch.equal(a, b) for a, b in zip(flat1, flat2))


@pytest.mark.parametrize("rdtype,bdtype", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                           (torch.bfloat16, torch.float16)])
@pytest.mark.parametrize("B,C,H,W", [(2, 96, 14, 14), (3, 30, 5, 7), (4, 768, 7, 7), (1, 2, 3, 3)])
def test_residual_add(rdtype, bdtype, B, C, H, W):
    """LayerScale residual add with a drop-path mask (utils/residual.py): the forward and every
    gradient against fp64 autograd; the mask's zero and 1/keep entries both occur."""
    from visionhope_b200.utils.residual import _VisionHOPEResidualFunction

    g = torch.Generator().manual_seed(B * 1000 + C + H)
    res = torch.randn(B, C, H, W, generator=g).to(rdtype).contiguous(memory_format=torch.channels_last)
    br = torch.randn(B, C, H, W, generator=g).to(bdtype).contiguous(memory_format=torch.channels_last)
    gamma = torch.randn(C, 1, 1, generator=g) * 0.5
    mask = torch.tensor([0.0, 1.25, 1.25, 0.0][:B] if B > 1 else [1.25])
    gout = torch.randn(B, C, H, W, generator=g)
    leaves = [t.to(DEV).requires_grad_(True) for t in (res, br, gamma)]
    out = _VisionHOPEResidualFunction.apply(*leaves, mask.to(DEV))
    assert out.dtype == torch.float32 and out.is_contiguous(memory_format=torch.channels_last)
    out.backward(gout.to(DEV))
    exp_out = og.residual(res.double(), br.double(), gamma.double(), mask.double())
    assert _rel(out, exp_out) < 1e-6
    exp = og.grads(og.residual, [res.float(), br.float(), gamma, mask], gout)
    assert leaves[0].grad.dtype == rdtype and _rel(leaves[0].grad, exp[0]) < _tol(rdtype)
    assert leaves[1].grad.dtype == bdtype and _rel(leaves[1].grad, exp[1]) < _tol(bdtype)
    assert leaves[2].grad.shape == gamma.shape and _rel(leaves[2].grad, exp[2]) < 2e-5


def test_residual_add_drop_path_and_determinism():
    """Outside training the mask is ones (the add is exact); in training the keep mask is
    drawn with bernoulli_ and divided by the keep probability; the backward repeats bit for bit."""
    from visionhope_b200.utils.residual import residual_add_backward, visionhope_residual_add

    g = torch.Generator().manual_seed(11)
    res = torch.randn(8, 64, 9, 9, generator=g).to(DEV).contiguous(memory_format=torch.channels_last)
    br = torch.randn(8, 64, 9, 9, generator=g).to(DEV).contiguous(memory_format=torch.channels_last)
    gamma = torch.randn(64, 1, 1, generator=g).to(DEV)
    out = visionhope_residual_add(res, br, gamma, 0.3, False)
    assert torch.equal(out, res + br * gamma)
    torch.manual_seed(5)
    out = visionhope_residual_add(res, br, gamma, 0.5, True)
    torch.manual_seed(5)
    mask = torch.empty((8,), device=DEV).bernoulli_(0.5).div_(0.5)
    assert torch.allclose(out, res + br * gamma * mask.view(-1, 1, 1, 1), rtol=1e-6, atol=1e-6)
    gout = torch.randn(8, 64, 9, 9, generator=g).to(DEV).contiguous(memory_format=torch.channels_last)
    r1 = residual_add_backward(gout, br, gamma, mask)
    r2 = residual_add_backward(gout, br, gamma, mask)
    assert all(torch.equal(a, b) for a, b in zip(r1, r2))


def test_srnl_backward_recompute_path_matches_full_history(monkeypatch):
    """head_dim 16 keeps the whole G history when it fits (the default here); with the history
    budget at 0 the backward recomputes each chunk's history instead.  Both give the same
    gradients (the same arithmetic in the same order)."""
    from visionhope_b200.srnl_core.chunk import sequence_backward

    mems, x, q, gy = _srnl_case(11, 2, 4, 2, 90, 16, False, False, torch.float32)
    args = ([m.to(DEV) for m in mems], x.to(DEV), q.to(DEV), [20] * 4, gy.to(DEV))
    full = sequence_backward(*args, q_normalized=False)
    monkeypatch.setenv("VHOPE_SRNL_BWD_HISTORY_BYTES", "0")
    rec = sequence_backward(*args, q_normalized=False)
    flat = lambda r: [*r[0], r[1], r[2]]
    assert all(torch.equal(a, b) for a, b in zip(flat(full), flat(rec)))
