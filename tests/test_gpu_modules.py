"""The reference's own modules (models/srnl.py, models/operator.py, unchanged) running over
this repository's drop-in modules on the GPU (``oracle/refmodel.py`` mode "dropin"): standalone
SRNL (config 1), the operator's ordinary, sequence and spatial paths, and the harness backbone
with CUDA-graph capture.  Kernel results are compared with the oracle on the exact tensors the
module fed the kernels (1e-4 normwise); the ordinary-vs-fused comparison under bf16 autocast
uses the north-star 2e-2 bar."""
import numpy as np
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _stress_(module, gen):
    """Non-default memories so the data-dependent gates are exercised."""
    with torch.no_grad():
        for p in module.initial_memories[:3]:
            p.copy_(torch.from_numpy(gen.normal(0, 0.3, tuple(p.shape)).astype(np.float32)))
        for p in module.initial_memories[3:]:
            p.copy_(torch.from_numpy(gen.normal(0, 0.6, tuple(p.shape)).astype(np.float32)))


def _scans(t):
    """[B, C, H, W] -> the four serialized scans [B, 4, L, C] as numpy fp32."""
    t = t.detach().float()
    hw = t.flatten(2).transpose(1, 2)
    wh = t.transpose(2, 3).flatten(2).transpose(1, 2)
    return torch.stack([hw, hw.flip(1), wh, wh.flip(1)], 1).cpu().numpy()


def _fusion_weights(op):
    return op.direction_weights().detach().float()


@pytest.mark.parametrize("fast", [False, True])
@pytest.mark.parametrize("kind", ["default", "stress"])
def test_standalone_srnl_config1(fast, kind, oracle, cuda, ref_dropin):
    """Config 1: SRNL(dim 64, head_dim 16, chunk 14), x [2, 196, 64] fp32."""
    torch.manual_seed(0)
    m = ref_dropin.SRNL(64, 16, chunk_size=14, fast_inference=fast).to(cuda).eval()
    if kind == "stress":
        _stress_(m, np.random.default_rng(0))
    x = torch.randn(2, 196, 64, device=cuda, generator=torch.Generator(cuda).manual_seed(0))
    with torch.no_grad():
        assert m.inference_status(x)["path"] == ("sequence" if fast else "ordinary")
        y = m(x)
    xp = x.view(2, 1, 196, 4, 16).transpose(2, 3).contiguous()
    exp = oracle.srnl_sequence([p.detach() for p in m.initial_memories], xp, x.unsqueeze(1), [14])
    exp = exp[:, 0].transpose(0, 2, 1, 3).reshape(2, 196, 64)
    assert y.shape == x.shape and y.dtype == torch.float32
    assert rel_err(y.cpu().numpy(), exp) < 1e-4


def test_srnl_rejects_cpu_and_bad_shapes(cuda, ref_dropin):
    SRNL = ref_dropin.SRNL
    m = SRNL(32, 16, directions=1)
    with pytest.raises(ValueError, match="same CUDA device"):
        m(torch.randn(1, 10, 32))
    m = m.to(cuda)
    with pytest.raises(ValueError, match="Standalone SRNL"):
        m(torch.randn(1, 10, 16, device=cuda))
    with pytest.raises(ValueError, match="nonempty"):
        m(torch.randn(0, 10, 32, device=cuda))
    with pytest.raises(ValueError):
        SRNL(30, 16)


def _operator(ref, C, gen, cuda, chunk=None, merge="scale", share=True):
    op = ref.VisionHOPEOperator(C, 16, chunk, merge, share).to(cuda).eval()
    _stress_(op.srnl, gen)
    with torch.no_grad():
        op.d_skip.normal_(0, 0.5)
        if op.direction_scale is not None:
            op.direction_scale.normal_(1, 0.3)
        if op.direction_logits is not None:
            op.direction_logits.normal_(0, 0.5)
    return op


def _oracle_operator(op, x, oracle):
    """Oracle of the operator on the exact x and W_q(x) the module sees (fp32 result, NCHW)."""
    B, C, H, W = x.shape
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        q = op.W_q(x.flatten(2).transpose(1, 2))
    qimg = q.transpose(1, 2).reshape(B, C, H, W)
    out = oracle.srnl_spatial([p.detach() for p in op.srnl.initial_memories], _scans(x), _scans(qimg),
                              op.d_skip.detach(), _fusion_weights(op), H, W, 16)
    return out.transpose(0, 3, 1, 2)


@pytest.mark.parametrize("merge,share", [("scale", True), ("softmax", False), ("sum", True)])
def test_operator_config2_ordinary_path(merge, share, oracle, cuda, ref_dropin):
    """Config 2 path: fp32 x under bf16 autocast -> qnorm + recurrence + fusion (ordinary)."""
    gen = np.random.default_rng(1)
    op = _operator(ref_dropin, 96, gen, cuda, merge=merge, share=share)
    op.fast_inference = True  # still ordinary: x fp32 vs bf16 queries (srnl.py:87-88)
    x = torch.randn(2, 96, 14, 14, device=cuda)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert op.inference_status(x)["path"] == "ordinary"
        y = op(x)
    assert y.dtype == torch.float32 and y.shape == x.shape
    assert rel_err(y.cpu().numpy(), _oracle_operator(op, x, oracle)) < 1e-4


@pytest.mark.parametrize("hw", [(14, 14), (9, 12), (28, 7)])
def test_operator_fast_spatial_path(hw, oracle, cuda, ref_dropin):
    gen = np.random.default_rng(2)
    op = _operator(ref_dropin, 64, gen, cuda)
    op.fast_inference = True
    H, W = hw
    x = torch.randn(3, 64, H, W, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert op.inference_status(x)["path"] == "spatial"
        y = op(x)
    assert y.is_contiguous(memory_format=torch.channels_last)
    assert rel_err(y.cpu().numpy(), _oracle_operator(op, x, oracle)) < 1e-4


def test_operator_fixed_chunk_sequence_path(oracle, cuda, ref_dropin):
    """chunk_size fixed and != H == W selects the sequence kernel + fusion (operator.py:141-152)."""
    gen = np.random.default_rng(3)
    op = _operator(ref_dropin, 32, gen, cuda, chunk=8)
    op.fast_inference = True
    x = torch.randn(2, 32, 12, 12, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert op.inference_status(x)["path"] == "sequence"
        y = op(x)
        q = op.project_queries(x.flatten(2).transpose(1, 2), 12, 12)
    xs = _scans(x)
    xp = xs.reshape(2, 4, 144, 2, 16).transpose(0, 1, 3, 2, 4).copy()
    ys = oracle.srnl_sequence([p.detach() for p in op.srnl.initial_memories], xp, q, [8] * 4)
    ys = torch.from_numpy(ys).to(torch.bfloat16).float().numpy()  # the sequence kernel stores bf16
    exp = oracle.dirfuse(ys, xp, op.d_skip.detach(), _fusion_weights(op), 12, 12, False)
    assert rel_err(y.float().cpu().numpy(), exp) < 1e-4


def test_fused_matches_ordinary_under_autocast(cuda, ref_dropin):
    """The reference's own ordinary-vs-fused parity: same bf16 input, both paths, 2e-2."""
    gen = np.random.default_rng(4)
    op = _operator(ref_dropin, 64, gen, cuda)
    x = torch.randn(2, 64, 14, 14, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        op.fast_inference = False
        ordinary = op(x)
        op.fast_inference = True
        fused = op(x)
    assert rel_err(fused.float().cpu().numpy(), ordinary.float().cpu().numpy()) < 2e-2


def test_rectangular_long_rows_ordinary_path(oracle, cuda, ref_dropin):
    """Config 5-like rows: W > 64 on the ordinary path (srnl_variable_lines)."""
    gen = np.random.default_rng(5)
    op = _operator(ref_dropin, 32, gen, cuda)
    x = torch.randn(1, 32, 6, 80, device=cuda).to(torch.bfloat16)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = op(x)
    exp = _oracle_operator(op, x, oracle)
    # the ordinary scans store y in bf16 before fusion
    assert rel_err(y.cpu().numpy(), exp) < 1e-2


def test_tiny_backbone_graph_and_paths(cuda):
    """The harness backbone: unprepared vs prepared under bf16 autocast, and CUDA-graph replay
    on changed inputs against eager (the reference's graph check, analysis/benchmark.py:74-87)."""
    from visionhope_b200.backbone import create_model, prepare_for_inference

    torch.manual_seed(3)
    model = create_model("visionhope_tiny").to(cuda).to(memory_format=torch.channels_last)
    x = torch.randn(2, 3, 224, 224, device=cuda).contiguous(memory_format=torch.channels_last)
    model.eval()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        ordinary = model(x).float()
    counts = prepare_for_inference(model)
    assert counts["srnl"] == 29 and counts["layerscale"] == 58 and counts["batchnorm_folded"] == 7
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        eager = model(x).float()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static = model(x)
        x.neg_().add_(0.125)
        g.replay()
        torch.cuda.synchronize()
        replay = static.float().clone()
        eager2 = model(x).float()
    assert torch.isfinite(eager).all()
    assert rel_err(eager.cpu().numpy(), ordinary.cpu().numpy()) < 2e-2
    torch.testing.assert_close(replay, eager2, atol=1e-3, rtol=1e-2)
