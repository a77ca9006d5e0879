"""The reference's own fused operator kernel against libvhope, side by side on one GPU.

The reference extension is built from the reference's sources by oracle/build_ref.py into
oracle/_ref (test infrastructure; the test skips when it was not built).  Both implementations
get the same bf16 inputs: the reference its four serialized scans [B, 4, L, C] (the layout its
operator materialises, models/operator.py:180-190), ours the one channels-last image.
Parity: fp32 outputs within 1e-4 normwise relative error.  The per-call device times are
printed (run with -s) as the per-kernel comparison; they are not asserted.
"""
import numpy as np
import pytest
import torch

from tests.conftest import make_memories, rel_err

pytestmark = pytest.mark.gpu


def _reference_extension():
    try:
        from oracle.build_ref import load_built

        return load_built("vhref_fused_bf16")
    except (FileNotFoundError, ImportError, OSError) as exc:
        pytest.skip(f"reference extension not built: {exc}")


def _time_ms(fn, iters=5):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / iters


SHAPES = [
    # (label, B, H, W, heads): the operator configuration (stage-1 shape, C = 96) and the
    # VisionHOPE-T stage-1 and stage-3 operators at batch 64
    ("operator-config", 64, 56, 56, 6),
    ("tiny-stage1", 64, 56, 56, 2),
    ("tiny-stage3", 64, 14, 14, 8),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s[0])
def test_reference_fused_operator_parity_and_time(shape, cuda):
    from visionhope_b200.srnl_core.fused import spatial_forward

    ext = _reference_extension()
    label, B, H, W, heads = shape
    D, C = 16, heads * 16
    gen = np.random.default_rng(5)
    mems = [torch.from_numpy(m).to(cuda) for m in make_memories(4, heads, D, "stress", gen)]
    img = torch.from_numpy(gen.normal(size=(B, H, W, C)).astype(np.float32)).to(cuda, torch.bfloat16)
    qimg = torch.from_numpy(gen.normal(size=(B, H, W, C)).astype(np.float32)).to(cuda, torch.bfloat16)
    skip = torch.from_numpy(gen.normal(0, 0.5, size=C).astype(np.float32)).to(cuda)
    wts = torch.from_numpy(gen.normal(1.0, 0.3, size=(4, C)).astype(np.float32)).to(cuda)

    def serialize(t):
        hw = t.reshape(B, H * W, C)
        wh = t.transpose(1, 2).reshape(B, H * W, C)
        return torch.stack([hw, hw.flip(1), wh, wh.flip(1)], dim=1).contiguous()

    xs, qs = serialize(img), serialize(qimg)
    ref = ext.srnl_line_forward_seq_noatomic(*mems, xs, qs, skip, wts, H, W, D)
    ours = spatial_forward(mems, img, qimg, skip, wts, H, W, D, layout="image")
    torch.cuda.synchronize()
    assert rel_err(ours.cpu().numpy(), ref.cpu().numpy()) < 1e-4

    t_ref = _time_ms(lambda: ext.srnl_line_forward_seq_noatomic(*mems, xs, qs, skip, wts, H, W, D))
    t_ref_e2e = _time_ms(lambda: ext.srnl_line_forward_seq_noatomic(*mems, serialize(img), serialize(qimg),
                                                                     skip, wts, H, W, D))
    t_ours = _time_ms(lambda: spatial_forward(mems, img, qimg, skip, wts, H, W, D, layout="image"))
    print(f"\n[{label}] B={B} {H}x{W} C={C}: reference kernel {t_ref:.3f} ms "
          f"(+ its scan materialisation {t_ref_e2e:.3f} ms), ours {t_ours:.3f} ms, "
          f"speed-up {t_ref / t_ours:.2f}x ({t_ref_e2e / t_ours:.2f}x with materialisation)")
