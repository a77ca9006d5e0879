"""GPU parity of the fused depthwise convolutions (vh_dwconv_fwd) against a float64 PyTorch
statement of the same arithmetic: convolution of the bf16-rounded input with bf16-rounded
weights and bias, the mode's epilogue, one rounding to the output dtype.  Tolerances: bf16
outputs within 4e-3 normwise (one bf16 rounding is <= 2^-9 relative), fp32 outputs 1e-5.
The GELU mode rounds its intermediate gelu(x) to bf16 (the dtype autocast gives it); the
kernel's erf (within 1.5e-7 of the exact one) moves that rounding for about 1 element in
5000, each by one bf16 step, so fp32 outputs of that mode are held to 1e-3."""
import zlib

import pytest
import torch
import torch.nn.functional as F

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@torch.no_grad()
def _expected(x, conv, mode, gate):
    bf = lambda t: t.to(torch.bfloat16).double()
    k = conv.kernel_size[0]
    xin = bf(x)
    if mode == "gelu":
        xin = bf(F.gelu(x.double()))
    conv_out = F.conv2d(xin, bf(conv.weight), bf(conv.bias), padding=k // 2, groups=x.shape[1])
    if mode == "bias":
        return conv_out
    if mode == "resid":
        return x.double() + conv_out
    if mode == "resid_add":
        s = x.double() + gate.double()
        s_conv = bf(s.to(x.dtype)) if x.dtype == torch.bfloat16 else bf(s)
        s_ref = s.to(x.dtype).double()
        return s_ref + F.conv2d(s_conv, bf(conv.weight), bf(conv.bias), padding=k // 2, groups=x.shape[1])
    if mode == "gate":
        return x.double() + torch.sigmoid(gate.double()) * conv_out
    return F.gelu(xin + conv_out)


CASES = [
    # (B, C, H, W, k, mode, dtype)
    (2, 64, 14, 14, 3, "resid", torch.float32),
    (2, 32, 56, 56, 7, "gate", torch.bfloat16),
    (3, 128, 14, 14, 5, "bias", torch.bfloat16),
    (2, 256, 7, 7, 3, "gelu", torch.bfloat16),
    (1, 40, 9, 13, 7, "gate", torch.bfloat16),    # channels not a multiple of 32, odd sizes
    (1, 8, 1, 17, 5, "bias", torch.float32),      # one row
    (2, 96, 23, 5, 3, "gelu", torch.float32),
    (1, 64, 33, 31, 7, "resid", torch.bfloat16),  # several 16 x 16 tiles with ragged edges
    (1, 512, 28, 28, 3, "gelu", torch.bfloat16),
    (1, 16, 16, 32, 5, "resid", torch.bfloat16),  # 16 x 16 tiles
    (2, 64, 28, 42, 7, "bias", torch.bfloat16),   # 14 x 14 tiles, several per image
    (1, 8, 7, 7, 7, "gate", torch.float32),       # kernel wider than half the image
    (2, 64, 14, 14, 3, "resid_add", torch.float32),   # cpe of x + a pending bf16 residual
    (1, 32, 9, 13, 3, "resid_add", torch.bfloat16),
    # 7 x 7 images run four whole images per CTA: batches that do not fill the last CTA,
    # channel counts that do not fill the last 32-channel group
    (5, 256, 7, 7, 3, "gelu", torch.bfloat16),
    (6, 40, 7, 7, 7, "gate", torch.bfloat16),
    (9, 32, 7, 7, 7, "gate", torch.float32),
    (5, 64, 7, 7, 5, "bias", torch.bfloat16),
    (2, 48, 7, 7, 3, "resid", torch.float32),
    (3, 96, 7, 7, 3, "resid_add", torch.float32),
    (7, 24, 7, 7, 3, "resid_add", torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(str(v).replace("torch.", "") for v in c))
def test_dwconv_matches_reference(case, cuda):
    from visionhope_b200.utils.dwconv import depthwise_fused

    B, C, H, W, k, mode, dt = case
    torch.manual_seed(zlib.crc32(repr(case).encode()))
    conv = torch.nn.Conv2d(C, C, k, padding=k // 2, groups=C).to(cuda)
    with torch.no_grad():
        conv.bias.normal_(0, 0.3)
    x = torch.randn(B, C, H, W, device=cuda).to(dt).contiguous(memory_format=torch.channels_last)
    gate = torch.randn_like(x) if mode == "gate" else None
    if mode == "resid_add":
        gate = torch.randn(x.shape, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode():
        if mode == "resid_add":
            y = depthwise_fused(x, conv, "resid", addend=gate)
        else:
            y = depthwise_fused(x, conv, mode, gate=gate)
    assert y.dtype == dt and y.shape == x.shape and y.is_contiguous(memory_format=torch.channels_last)
    exp = _expected(x, conv, mode, gate)
    tol = 4e-3 if dt == torch.bfloat16 else (1e-3 if mode == "gelu" else 1e-5)
    assert rel_err(y.float().cpu().numpy(), exp.cpu().numpy()) < tol


def test_dwconv_fusable_rules(cuda):
    from visionhope_b200.utils.dwconv import fusable

    conv = torch.nn.Conv2d(16, 16, 3, padding=1, groups=16).to(cuda)
    x = torch.randn(1, 16, 8, 8, device=cuda).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode():
        assert not fusable(x, conv)  # no autocast: fp32 convolution arithmetic stays with PyTorch
        with torch.autocast("cuda", dtype=torch.bfloat16):
            assert fusable(x, conv)
            assert not fusable(x.contiguous(), conv)
            assert not fusable(x, torch.nn.Conv2d(16, 16, 3, padding=1, groups=16, bias=False).to(cuda))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        assert not fusable(x, conv)  # autograd on


def test_dwconv_rejects_bad_arguments(cuda):
    from visionhope_b200.utils.dwconv import depthwise_fused

    conv = torch.nn.Conv2d(12, 12, 3, padding=1, groups=12).to(cuda)
    x = torch.randn(1, 12, 8, 8, device=cuda).contiguous(memory_format=torch.channels_last)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        depthwise_fused(x, conv, "bias")
    conv = torch.nn.Conv2d(16, 16, 3, padding=1, groups=16).to(cuda)
    x = torch.randn(1, 16, 8, 8, device=cuda).contiguous(memory_format=torch.channels_last)
    with pytest.raises(RuntimeError, match="gate"):
        depthwise_fused(x, conv, "gate")


@pytest.mark.parametrize("shape", [(2, 256, 56, 56), (3, 1024, 14, 14), (2, 2048, 7, 7), (5, 2048, 7, 7),
                                   (6, 40, 7, 7), (1, 96, 23, 5), (2, 512, 28, 28)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_dwconv_gelu_tile_sums(shape, dt, cuda):
    """The GELU epilogue's per-tile sums of y^2 (the statistics of the GRN that follows): y is
    unchanged by asking for them, the tiles add up to the image's per-channel sums of y as
    stored, and tile 0 of a 56 x 56 image is its top-left 14 x 14 block."""
    from visionhope_b200 import _lib
    from visionhope_b200.utils.dwconv import depthwise_fused

    B, C, H, W = shape
    torch.manual_seed(zlib.crc32(repr(shape).encode()))
    conv = torch.nn.Conv2d(C, C, 3, padding=1, groups=C).to(cuda)
    x = torch.randn(B, C, H, W, device=cuda).to(dt).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode():
        y0 = depthwise_fused(x, conv, "gelu")
        y, ss = depthwise_fused(x, conv, "gelu", with_sumsq=True)
    assert torch.equal(y, y0)
    assert ss.shape == (B, _lib.load().vh_dwconv_tiles(H, W), C) and ss.dtype == torch.float32
    yd = y.double()
    exp = yd.pow(2).sum(dim=(2, 3))
    assert rel_err(ss.double().sum(1).cpu().numpy(), exp.cpu().numpy()) < 1e-6
    if H == W == 56:
        assert rel_err(ss[:, 0].double().cpu().numpy(), yd[:, :, :14, :14].pow(2).sum(dim=(2, 3)).cpu().numpy()) < 1e-6


@pytest.mark.parametrize("shape", [(5, 128, 14, 14), (3, 40, 14, 14), (6, 256, 7, 7), (3, 24, 7, 7)],
                         ids=lambda s: "x".join(map(str, s)))
def test_dwconv_gate_pos_matches_gate_then_bias(shape, cuda):
    """The fused local features + output position term ("gate_pos") is bit-identical to the
    gated 7x7 call followed by the 5x5 bias call on its output (same operands, same order of
    sums), for whole 14 x 14 images and four 7 x 7 images per CTA, with batches and channel
    counts that leave CTAs partly empty."""
    from visionhope_b200.utils.dwconv import depthwise_fused, gate_pos_ok

    B, C, H, W = shape
    torch.manual_seed(zlib.crc32(repr(shape).encode()))
    conv, pos = (torch.nn.Conv2d(C, C, 7, padding=3, groups=C).to(cuda),
                 torch.nn.Conv2d(C, C, 5, padding=2, groups=C).to(cuda))
    with torch.no_grad():
        conv.bias.normal_(0, 0.3)
        pos.bias.normal_(0, 0.3)
    x = torch.randn(B, C, H, W, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    gate = torch.randn_like(x)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert gate_pos_ok(x, conv, pos)
        y, p = depthwise_fused(x, conv, "gate_pos", gate=gate, pos_conv=pos)
        y0 = depthwise_fused(x, conv, "gate", gate=gate)
        p0 = depthwise_fused(y0, pos, "bias")
    assert torch.equal(y, y0)
    assert torch.equal(p, p0)
    assert rel_err(p.double().cpu().numpy(), _expected(y0, pos, "bias", None).cpu().numpy()) < 4e-3


def test_dwconv_gate_pos_rejects_other_shapes(cuda):
    from visionhope_b200.utils.dwconv import depthwise_fused, gate_pos_ok

    conv = torch.nn.Conv2d(32, 32, 7, padding=3, groups=32).to(cuda)
    pos = torch.nn.Conv2d(32, 32, 5, padding=2, groups=32).to(cuda)
    x = torch.randn(1, 32, 28, 28, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert not gate_pos_ok(x, conv, pos)
        with pytest.raises(RuntimeError):
            depthwise_fused(x, conv, "gate_pos", gate=torch.randn_like(x), pos_conv=pos)


def test_dwconv_sumsq_needs_gelu(cuda):
    from visionhope_b200.utils.dwconv import depthwise_fused

    conv = torch.nn.Conv2d(16, 16, 3, padding=1, groups=16).to(cuda)
    x = torch.randn(1, 16, 8, 8, device=cuda).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), pytest.raises(RuntimeError, match="gelu"):
        depthwise_fused(x, conv, "bias", with_sumsq=True)
