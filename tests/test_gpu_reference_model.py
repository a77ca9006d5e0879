"""Parity against the reference itself, on the configurations the headline rests on.

The reference's own modules (``oracle/refmodel.py``) run in two modes: "native" on the
reference's own kernels (built from its sources by ``oracle/build_ref.py``) and "dropin" over
this repository's modules.  Each test runs every native computation before it imports the
drop-in mode (the reference's modules resolve their kernel modules at call time).

* VisionHOPE-T, 224 x 224, batch 8, bf16 autocast, prepared (config 4's model): the logits of
  the harness backbone (``visionhope_b200.backbone``, same state_dict) and of the drop-in run
  against the native run within 2e-2 normwise; every operator of the native run re-run on its
  captured input by this repository's scan launch, within 1e-4 (same queries) -- LayerScale
  1e-6 would hide an operator error in the logits.  A second state with LayerScale 0.1 and
  data-dependent SRNL gates makes every block matter.
* Config 2 at its own shape: VisionHOPEOperator(96) at B=64, 56 x 56, fp32 x under bf16
  autocast (the ordinary path: qnorm, chunk forward, direction fusion) -- native, drop-in and
  the CPU oracle on the exact inputs, all within 1e-4.
* The dense-prediction adapter (tasks/backbone.py ``VisionHOPEBackbone``, with its per-stage
  output norms) against ``visionhope_b200.backbone.DenseBackbone`` on one state_dict, measured
  against the reference's own fp32 run.
* VisionHOPE-B's stage-1 operator at the dense configuration's shape (config 5): B=2,
  C=48, 128 x 512 tokens (row chunks of 512, column chunks of 128), bf16, on the fast spatial
  path (1e-4 against native and oracle) and on the ordinary path (``srnl_variable_lines``,
  which stores y in bf16: 1e-2).
Device times of the reference and of this repository are printed (run with -s).
"""
import numpy as np
import pytest
import torch

from tests.conftest import reference, rel_err

pytestmark = pytest.mark.gpu


def _time_ms(fn, iters=3):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / iters


def _stress_memories(model, gen):
    with torch.no_grad():
        for name, p in model.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            if leaf in ("M_m_0", "M_v_0", "M_k_0"):
                p.copy_(torch.from_numpy(gen.normal(0, 0.3, tuple(p.shape)).astype(np.float32)))
            elif leaf in ("M_eta_0", "M_alpha_0"):
                p.copy_(torch.from_numpy(gen.normal(0, 0.6, tuple(p.shape)).astype(np.float32)))
            elif leaf == "d_skip":
                p.normal_(0, 0.5)


def _blocks(model):
    return [m for m in model.modules() if type(m).__name__ == "VisionHOPEBlock"]


def _capture_fast_operators(model, records):
    """Record (x_local, fp32 NHWC output) of every operator's fused call (block.py:73-80)."""
    for blk in _blocks(model):
        op = blk.operator

        def wrapped(x, path, _orig=op._forward_fast):
            out = _orig(x, path)
            records.append((x.detach().clone(), out.detach().clone()))
            return out
        op._forward_fast = wrapped


def _fresh_state(ref, name, layer_scale, stress):
    torch.manual_seed(3)
    kw = {} if layer_scale is None else {"layer_scale_init_value": layer_scale}
    m = ref.create_model(name, **kw)
    if stress:
        _stress_memories(m, np.random.default_rng(7))
    return {k: v.detach().clone() for k, v in m.state_dict().items()}, kw


def _run_reference_model(ref, name, sd, kw, x, records=None):
    model = ref.create_model(name, **kw)
    model.load_state_dict(sd, strict=True)
    model = model.cuda().to(memory_format=torch.channels_last)
    ref.prepare_for_inference(model)
    if records is not None:
        _capture_fast_operators(model, records)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(x).float()
        ms = _time_ms(lambda: model(x))
    return logits, ms, model


@pytest.mark.parametrize("layer_scale,stress", [(None, False), (0.1, True)], ids=["default", "stress"])
def test_visionhope_tiny_logits_match_reference(layer_scale, stress, cuda):
    from visionhope_b200.backbone import create_model, prepare_for_inference
    from visionhope_b200.srnl_core.fused import spatial_forward

    native = reference("native")
    sd, kw = _fresh_state(native, "visionhope_tiny", layer_scale, stress)
    x = torch.randn(8, 3, 224, 224, generator=torch.Generator().manual_seed(3)).to(cuda)
    x = x.contiguous(memory_format=torch.channels_last)
    records = []
    ref_logits, ref_ms, ref_model = _run_reference_model(native, "visionhope_tiny", sd, kw, x, records)
    ops = [blk.operator for blk in _blocks(ref_model)]
    assert len(ops) == 29 and len(records) >= 29
    records = records[:29]

    # every operator of the reference run, re-run by this repository's scan launch on the same
    # x_local and the same queries (W_q as the reference's project_queries computes it)
    worst = 0.0
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        for op, (xl, out_ref) in zip(ops, records):
            B, C, H, W = xl.shape
            q = op.W_q(xl.flatten(2).transpose(1, 2)).reshape(B, H, W, C)
            ours = spatial_forward(op.srnl.initial_memories, xl.permute(0, 2, 3, 1), q, op.d_skip,
                                   op.direction_weights().float(), H, W, op.head_dim, layout="image")
            worst = max(worst, rel_err(ours, out_ref))
    assert worst < 1e-4, worst

    model = create_model("visionhope_tiny", **kw)
    model.load_state_dict(sd, strict=True)
    model = model.cuda().to(memory_format=torch.channels_last)
    prepare_for_inference(model)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        ours_logits = model(x).float()
        ours_ms = _time_ms(lambda: model(x))
    del model, ref_model

    dropin = reference("dropin")
    drop_logits, drop_ms, _ = _run_reference_model(dropin, "visionhope_tiny", sd, kw, x)
    e_harness = rel_err(ours_logits, ref_logits)
    e_dropin = rel_err(drop_logits, ref_logits)
    print(f"\n[visionhope_tiny {'stress' if stress else 'default'}] logits rel err: harness {e_harness:.2e}, "
          f"drop-in {e_dropin:.2e}; worst operator {worst:.2e}; batch 8 eager forward: reference "
          f"{ref_ms:.2f} ms, drop-in {drop_ms:.2f} ms, harness {ours_ms:.2f} ms")
    assert torch.isfinite(ref_logits).all()
    assert e_harness < 2e-2 and e_dropin < 2e-2


def _config2_operator(ref, sd=None):
    torch.manual_seed(1)
    op = ref.VisionHOPEOperator(96, 16, None, "scale", True)
    if sd is None:
        _stress_memories(op, np.random.default_rng(1))
        with torch.no_grad():
            op.direction_scale.normal_(1, 0.3)
        sd = {k: v.detach().clone() for k, v in op.state_dict().items()}
    else:
        op.load_state_dict(sd)
    op = op.cuda().eval()
    op.fast_inference = True  # still the ordinary path: fp32 x, bf16 queries (srnl.py:87-88)
    return op, sd


def _scans(t):
    t = t.detach().float()
    hw = t.flatten(2).transpose(1, 2)
    wh = t.transpose(2, 3).flatten(2).transpose(1, 2)
    return torch.stack([hw, hw.flip(1), wh, wh.flip(1)], 1).cpu().numpy()


def test_config2_operator_full_shape_ordinary_path(oracle, cuda):
    """B=64, C=96, 56 x 56, fp32 x ~ N(0,1) (seed 1) under bf16 autocast."""
    x = torch.randn(64, 96, 56, 56, generator=torch.Generator().manual_seed(1)).to(cuda)
    native = reference("native")
    op, sd = _config2_operator(native)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert op.inference_status(x)["path"] == "ordinary"
        y_ref = op(x)
        t_ref = _time_ms(lambda: op(x))
        q = op.W_q(x.flatten(2).transpose(1, 2))
    qimg = q.transpose(1, 2).reshape(x.shape)
    exp = oracle.srnl_spatial([p.detach() for p in op.srnl.initial_memories], _scans(x), _scans(qimg),
                              op.d_skip.detach(), op.direction_weights().detach().float(), 56, 56, 16)
    exp = exp.transpose(0, 3, 1, 2)
    y_ref = y_ref.cpu()
    del op

    dropin = reference("dropin")
    op, _ = _config2_operator(dropin, sd)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = op(x)
        t_ours = _time_ms(lambda: op(x))
    e_ours, e_ref, e_pair = rel_err(y, exp), rel_err(y_ref, exp), rel_err(y, y_ref)
    print(f"\n[config 2, ordinary path] rel err vs oracle: ours {e_ours:.2e}, reference {e_ref:.2e}; "
          f"ours vs reference {e_pair:.2e}; operator call: reference {t_ref:.2f} ms, ours {t_ours:.2f} ms")
    assert y.dtype == torch.float32 and y.shape == x.shape
    assert e_ours < 1e-4 and e_ref < 1e-4 and e_pair < 1e-4


def _config5_stage1(ref, sd=None):
    torch.manual_seed(4)
    op = ref.VisionHOPEOperator(48, 16, None, "scale", True)
    if sd is None:
        _stress_memories(op, np.random.default_rng(4))
        sd = {k: v.detach().clone() for k, v in op.state_dict().items()}
    else:
        op.load_state_dict(sd)
    return op.cuda().eval(), sd


@pytest.mark.parametrize("fast", [True, False], ids=["fast", "ordinary"])
def test_config5_stage1_operator_128x512(fast, oracle, cuda):
    """VisionHOPE-B stage 1 at 512 x 2048 input: [2, 48, 128, 512] bf16 channels-last."""
    x = torch.randn(2, 48, 128, 512, generator=torch.Generator().manual_seed(4)).to(cuda, torch.bfloat16)
    x = x.contiguous(memory_format=torch.channels_last)
    native = reference("native")
    op, sd = _config5_stage1(native)
    op.fast_inference = fast
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert op.inference_status(x)["path"] == ("spatial" if fast else "ordinary")
        y_ref = op(x).float()
        t_ref = _time_ms(lambda: op(x))
        q = op.W_q(x.flatten(2).transpose(1, 2))
    qimg = q.transpose(1, 2).reshape(x.shape)
    exp = oracle.srnl_spatial([p.detach() for p in op.srnl.initial_memories], _scans(x), _scans(qimg),
                              op.d_skip.detach(), op.direction_weights().detach().float(), 128, 512, 16)
    exp = exp.transpose(0, 3, 1, 2)
    y_ref = y_ref.cpu()
    del op

    dropin = reference("dropin")
    op, _ = _config5_stage1(dropin, sd)
    op.fast_inference = fast
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = op(x).float()
        t_ours = _time_ms(lambda: op(x))
    tol = 1e-4 if fast else 1e-2  # the ordinary scans store y in bf16 before the fusion
    e_ours, e_ref, e_pair = rel_err(y, exp), rel_err(y_ref, exp), rel_err(y, y_ref)
    print(f"\n[config 5 stage 1, {'fast' if fast else 'ordinary'}] rel err vs oracle: ours {e_ours:.2e}, "
          f"reference {e_ref:.2e}; ours vs reference {e_pair:.2e}; operator call: reference {t_ref:.2f} ms, "
          f"ours {t_ours:.2f} ms")
    assert e_ours < tol and e_ref < tol and e_pair < tol


def test_dense_backbone_matches_reference(cuda):
    """tasks/backbone.py's VisionHOPEBackbone (the reference's adapter for Mask R-CNN and
    UPerNet, unchanged, on its own kernels) against DenseBackbone with its state_dict:
    VisionHOPE-T, 2 x 3 x 256 x 384 (stage 1: 64 x 96 tokens), prepared, output norms with
    non-trivial weights, LayerScale 0.1 and stressed SRNL memories (every block matters).

    The normalized stage features of a bf16-autocast run drift from an fp32 run by about 2e-2
    after a few such blocks, whichever kernels run, so the bar is relative to the reference's own
    drift: against the reference's fp32 run, ours (bf16) must be within 1.5x of the reference's
    bf16 run (floor 1e-2), and within 4e-2 of the reference's bf16 run itself."""
    import importlib

    from visionhope_b200.backbone import DenseBackbone, prepare_for_inference

    native = reference("native")
    tb = importlib.import_module("visionhope.tasks.backbone")
    torch.manual_seed(4)
    ref_bb = tb.VisionHOPEBackbone("tiny", layer_scale_init_value=0.1)
    _stress_memories(ref_bb, np.random.default_rng(5))
    with torch.no_grad():
        for n in ref_bb.out_norms:
            n.weight.normal_(1, 0.2)
            n.bias.normal_(0, 0.2)
    sd = {k: v.detach().clone() for k, v in ref_bb.state_dict().items()}
    ref_bb = ref_bb.cuda().to(memory_format=torch.channels_last)
    native.prepare_for_inference(ref_bb)
    x = torch.randn(2, 3, 256, 384, generator=torch.Generator().manual_seed(6)).to(cuda)
    with torch.inference_mode():
        ref32 = [o.float() for o in ref_bb(x)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            ref16 = [o.float() for o in ref_bb(x)]
            ref_ms = _time_ms(lambda: ref_bb(x))
    del ref_bb

    ours = DenseBackbone("tiny", layer_scale_init_value=0.1)
    ours.load_state_dict(sd, strict=True)
    ours = ours.cuda().to(memory_format=torch.channels_last)
    prepare_for_inference(ours)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        our16 = [o.float() for o in ours(x)]
        our_ms = _time_ms(lambda: ours(x))
    assert len(our16) == len(ref16) == len(ref32) == 4
    e_ref = [rel_err(a, t) for a, t in zip(ref16, ref32)]
    e_our = [rel_err(b, t) for b, t in zip(our16, ref32)]
    e_pair = [rel_err(b, a) for a, b in zip(ref16, our16)]
    fmt = lambda v: " ".join(f"{e:.2e}" for e in v)
    print(f"\n[dense backbone] vs fp32 reference: reference bf16 {fmt(e_ref)}; ours bf16 {fmt(e_our)}; "
          f"ours vs reference bf16 {fmt(e_pair)}; eager bf16 forward reference {ref_ms:.2f} ms, ours {our_ms:.2f} ms")
    for a, b, t in zip(ref16, our16, ref32):
        assert a.shape == b.shape == t.shape and torch.isfinite(b).all()
    for er, eo, ep in zip(e_ref, e_our, e_pair):
        assert eo < max(1e-2, 1.5 * er), (e_ref, e_our)
        assert ep < 4e-2, e_pair
