"""GPU parity of query normalization, direction fusion, GRN and LayerNorm against the oracle
(fp32 outputs: 1e-4 normwise relative error; these are pure-fp32 arithmetic kernels)."""
import zlib

import numpy as np
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _dev(a, dev, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev, dt)


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("D", [4, 16, 64])
def test_qnorm(dt, D, oracle, cuda):
    from visionhope_b200.utils.query_normalization import visionhope_qnorm

    gen = np.random.default_rng(D)
    B, L, heads = 2, 37, 3
    q = _dev(gen.normal(size=(B, 4, L, heads * D)), cuda, DT[dt])
    q[0, 1, 3] = 0  # an all-zero query row hits the 1e-12 floor
    out = visionhope_qnorm(q, heads, D)
    exp, _ = oracle.qnorm(q, heads, D)
    assert out.dtype == torch.float32 and tuple(out.shape) == (B, 4, heads, L, D)
    assert rel_err(out.cpu().numpy(), exp) < 1e-6


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("channels_last", [False, True])
@pytest.mark.parametrize("per_dir", [False, True])
def test_direction_fusion(dt, channels_last, per_dir, oracle, cuda):
    from visionhope_b200.utils.direction_fusion import visionhope_postprocess_scale

    gen = np.random.default_rng(3)
    B, heads, H, W, D = 2, 3, 9, 13, 16
    C = heads * D
    y = _dev(gen.normal(size=(B, 4, heads, H * W, D)), cuda, DT[dt])
    x = _dev(gen.normal(size=(B, 4, heads, H * W, D)), cuda, DT[dt])
    skip = _dev(gen.normal(size=(4, heads, D) if per_dir else (heads, D)), cuda)
    scale = _dev(gen.normal(1, 0.3, size=(4, C)), cuda)
    out = visionhope_postprocess_scale(y, x, skip, scale, H, W, channels_last)
    exp = oracle.dirfuse(y, x, skip, scale, H, W, False)
    assert out.shape == (B, C, H, W)
    assert out.is_contiguous(memory_format=torch.channels_last if channels_last else torch.contiguous_format)
    assert rel_err(out.cpu().numpy(), exp) < 1e-6


GRN_CASES = [(4, 14, 14, 96, "f32"), (3, 7, 7, 768, "bf16"), (2, 5, 3, 2048, "f16"),
             (1, 56, 56, 32, "bf16"), (6, 1, 1, 12, "f32"), (2, 9, 9, 4100, "f32"),
             (2, 56, 56, 256, "bf16"),   # stage-1 FFN width: a 16-CTA cluster per image
             (2, 6, 6, 12, "bf16"),      # rows not 16-byte multiples: two-pass kernels
             (1, 128, 128, 256, "f32")]  # image beyond any cluster's shared memory: two-pass


@pytest.mark.parametrize("case", GRN_CASES, ids=lambda c: "x".join(map(str, c)))
def test_grn(case, oracle, cuda):
    from visionhope_b200.utils.grn import global_response_norm

    B, H, W, C, dt = case
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    x_nhwc = gen.normal(size=(B, H, W, C))
    x = _dev(x_nhwc, cuda, DT[dt]).permute(0, 3, 1, 2)  # channels-last logical NCHW
    gamma = _dev(gen.normal(0, 0.02, size=(1, C, 1, 1)), cuda)
    beta = _dev(gen.normal(0, 0.02, size=(1, C, 1, 1)), cuda)
    y = global_response_norm(x, gamma, beta)
    exp = oracle.grn_nhwc(x.permute(0, 2, 3, 1), gamma, beta)
    assert y.dtype == torch.float32 and y.is_contiguous(memory_format=torch.channels_last)
    assert rel_err(y.permute(0, 2, 3, 1).cpu().numpy(), exp) < 1e-5


def test_grn_stats_outputs(oracle, cuda):
    from visionhope_b200.utils.grn_cuda import grn_forward

    gen = np.random.default_rng(9)
    x = _dev(gen.normal(size=(3, 10, 10, 64)), cuda).permute(0, 3, 1, 2)
    g, b = _dev(gen.normal(size=64), cuda), _dev(gen.normal(size=64), cuda)
    _, gx, inv = grn_forward(x, g, b, 1e-6, want_stats=True)
    xn = x.permute(0, 2, 3, 1).double().cpu()
    gx_exp = xn.pow(2).sum(dim=(1, 2)).sqrt()
    assert torch.allclose(gx.double().cpu(), gx_exp, rtol=1e-5)
    assert torch.allclose(inv.double().cpu(), 1.0 / (gx_exp.mean(1) + 1e-6), rtol=1e-5)


LN_CASES = [(4, 14, 14, 96, "f32"), (3, 7, 7, 768, "bf16"), (2, 56, 56, 64, "bf16"),
            (2, 5, 5, 32, "f16"), (2, 3, 3, 2048, "f32"), (2, 4, 4, 100, "f32"),
            (1, 3, 3, 4099, "bf16"), (1, 2, 2, 30, "f32"), (1, 3, 7, 64, "f32"),
            (3, 5, 7, 256, "f32"), (1, 1, 1, 8, "bf16")]


@pytest.mark.parametrize("case", LN_CASES, ids=lambda c: "x".join(map(str, c)))
def test_layernorm(case, oracle, cuda):
    from visionhope_b200.utils.layer_norm_cuda import visionhope_layernorm2d

    B, H, W, C, dt = case
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    x = _dev(gen.normal(size=(B, H, W, C)) * 3 + 1, cuda, DT[dt]).permute(0, 3, 1, 2)
    w = _dev(gen.normal(1, 0.02, size=C), cuda)
    b = _dev(gen.normal(0, 0.02, size=C), cuda)
    y = visionhope_layernorm2d(x, w, b, 1e-6)
    exp = oracle.layernorm_rows(x.permute(0, 2, 3, 1).reshape(-1, C), w, b)
    assert y.dtype == torch.float32 and y.shape == (B, C, H, W)
    assert rel_err(y.permute(0, 2, 3, 1).reshape(-1, C).cpu().numpy(), exp) < 1e-5


@pytest.mark.parametrize("out", ["bf16", "f16"])
def test_norms_emit_half_outputs(out, oracle, cuda):
    """GRN and LN written in a 16-bit dtype equal their fp32 result rounded once."""
    from visionhope_b200.utils.grn_cuda import grn_forward
    from visionhope_b200.utils.layer_norm_cuda import layernorm_rows

    gen = np.random.default_rng(11)
    x = _dev(gen.normal(size=(2, 28, 28, 512)), cuda, torch.bfloat16).permute(0, 3, 1, 2)
    g, b = _dev(gen.normal(0, 0.02, size=512), cuda), _dev(gen.normal(0, 0.02, size=512), cuda)
    y32 = grn_forward(x, g, b, 1e-6)
    y16 = grn_forward(x, g, b, 1e-6, out_dtype=DT[out])
    assert y16.dtype == DT[out] and torch.equal(y16, y32.to(DT[out]))
    rows = _dev(gen.normal(size=(777, 256)) * 2, cuda)
    w, bb = _dev(gen.normal(1, 0.02, size=256), cuda), _dev(gen.normal(0, 0.02, size=256), cuda)
    l32 = layernorm_rows(rows, w, bb, 1e-6)
    l16 = layernorm_rows(rows, w, bb, 1e-6, out_dtype=DT[out])
    assert l16.dtype == DT[out] and torch.equal(l16, l32.to(DT[out]))


@pytest.mark.parametrize("xdt,rdt,ydt", [("f32", "bf16", "bf16"), ("f32", "f32", "f32"), ("bf16", "bf16", "bf16")])
def test_add_layernorm(xdt, rdt, ydt, oracle, cuda):
    """s = x + r stored in x's dtype and LayerNorm of the stored s, against the oracle."""
    from visionhope_b200.utils.layer_norm_cuda import add_layernorm_rows, layernorm_rows

    gen = np.random.default_rng(13)
    for rows, C in ((777, 64), (1000, 256), (33, 512)):
        x = _dev(gen.normal(size=(rows, C)), cuda, DT[xdt])
        r = _dev(gen.normal(size=(rows, C)), cuda, DT[rdt])
        w = _dev(gen.normal(1, 0.02, size=C), cuda)
        b = _dev(gen.normal(0, 0.02, size=C), cuda)
        s_exp = (x.float() + r.float()).to(DT[xdt])
        s, y = add_layernorm_rows(x.clone(), r, w, b, 1e-6, out_dtype=DT[ydt])
        assert torch.equal(s, s_exp)
        exp = oracle.layernorm_rows(s_exp.float(), w, b)
        tol = 1e-5 if ydt == "f32" else 4e-3
        assert rel_err(y.float().cpu().numpy(), exp) < tol
        # in place into x
        x2 = x.clone()
        s2, y2 = add_layernorm_rows(x2, r, w, b, 1e-6, out_dtype=DT[ydt])
        assert s2.data_ptr() == x2.data_ptr() and torch.equal(x2, s_exp) and torch.equal(y2, y)


@pytest.mark.parametrize("act", [None, "gelu"])
@pytest.mark.parametrize("io", [("bf16", "bf16"), ("bf16", "f32"), ("f32", "f32")])
def test_bias_act(act, io, cuda):
    """act(x + b) in fp32, rounded once: against float64 PyTorch (exact erf GELU)."""
    import torch.nn.functional as F

    from visionhope_b200.utils.bias_act import bias_act

    gen = np.random.default_rng(17)
    x = _dev(gen.normal(size=(3, 9, 11, 48)) * 2, cuda, DT[io[0]]).permute(0, 3, 1, 2)
    b = _dev(gen.normal(size=48), cuda)
    y = bias_act(x, b, act, out_dtype=DT[io[1]])
    exp = x.double() + b.double().view(1, -1, 1, 1)
    if act == "gelu":
        exp = F.gelu(exp)
    assert y.dtype == DT[io[1]] and y.is_contiguous(memory_format=torch.channels_last)
    tol = 4e-3 if io[1] == "bf16" else 1e-6
    assert rel_err(y.double().cpu().numpy(), exp.cpu().numpy()) < tol


GRN_APPLY_CASES = [(2, 56, 56, 256, "bf16", 16), (3, 14, 14, 1024, "bf16", 1), (2, 7, 7, 2048, "f32", 1),
                   (4, 9, 9, 64, "f16", 3), (1, 5, 5, 8, "f32", 2), (2, 28, 28, 512, "bf16", 4),
                   (3, 56, 56, 96, "f32", 1), (2, 7, 7, 768, "bf16", 2), (1, 3, 5, 24, "f32", 1)]


@pytest.mark.parametrize("case", GRN_APPLY_CASES, ids=lambda c: "x".join(map(str, c)))
def test_grn_apply_from_slice_sums(case, oracle, cuda):
    """GRN fed with per-slice sums of x^2 (as the fused depthwise GELU kernel produces them)
    against the oracle's GRN of the same x."""
    from visionhope_b200.utils.grn_cuda import grn_apply

    B, H, W, C, dt, P = case
    gen = np.random.default_rng(zlib.crc32(repr(case).encode()))
    x = _dev(gen.normal(size=(B, H, W, C)), cuda, DT[dt]).permute(0, 3, 1, 2)
    gamma = _dev(gen.normal(0, 0.5, size=C), cuda)
    beta = _dev(gen.normal(0, 0.5, size=C), cuda)
    xs = x.permute(0, 2, 3, 1).reshape(B, H * W, C).double().cpu()
    bounds = np.linspace(0, H * W, P + 1).astype(int)
    sums = torch.stack([xs[:, a:b].pow(2).sum(1) for a, b in zip(bounds[:-1], bounds[1:])], 1)
    y = grn_apply(x, sums.float().to(cuda), gamma, beta, 1e-6)
    exp = oracle.grn_nhwc(x.permute(0, 2, 3, 1), gamma, beta)
    assert y.dtype == torch.float32 and y.is_contiguous(memory_format=torch.channels_last)
    assert rel_err(y.permute(0, 2, 3, 1).cpu().numpy(), exp) < 1e-5
    yb = grn_apply(x, sums.float().to(cuda), gamma, beta, 1e-6, out_dtype=torch.bfloat16)
    assert rel_err(yb.float().permute(0, 2, 3, 1).cpu().numpy(), exp) < 1e-2


def test_grn_apply_rejects_unsupported_channels(cuda):
    from visionhope_b200.utils.grn_cuda import grn_apply, grn_apply_ok

    for C in (12, 20, 4096):
        x = torch.zeros(1, C, 2, 2, device=cuda).contiguous(memory_format=torch.channels_last)
        assert not grn_apply_ok(x)
        g = torch.zeros(C, device=cuda)
        with pytest.raises(RuntimeError, match="channels"):
            grn_apply(x, torch.zeros(1, 1, C, device=cuda), g, g, 1e-6)


@pytest.mark.parametrize("xdt,rdt,ydt", [(torch.float32, torch.bfloat16, torch.bfloat16),
                                         (torch.float32, torch.float32, torch.float32),
                                         (torch.bfloat16, torch.bfloat16, torch.float32)])
def test_add_cast(xdt, rdt, ydt, cuda):
    """(y dtype)(x + r) summed in fp32 and rounded once: bit-exact against torch's fp32 add
    followed by the cast."""
    from visionhope_b200.utils.bias_act import add_cast

    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(3, 64, 9, 7, device=cuda, generator=g).to(xdt).contiguous(memory_format=torch.channels_last)
    r = torch.randn(3, 64, 9, 7, device=cuda, generator=g).to(rdt).contiguous(memory_format=torch.channels_last)
    y = add_cast(x, r, ydt)
    assert y.dtype == ydt and y.is_contiguous(memory_format=torch.channels_last)
    assert torch.equal(y, (x.float() + r.float()).to(ydt))
    with pytest.raises(RuntimeError):
        add_cast(x, r.contiguous(), ydt)


@pytest.mark.parametrize("cout,H,W,act,ydt", [(32, 224, 224, "gelu", torch.bfloat16), (48, 37, 50, "gelu", torch.bfloat16),
                                              (16, 9, 7, None, torch.float32), (64, 64, 66, "gelu", torch.float32)])
def test_stem_conv(cout, H, W, act, ydt, cuda):
    """First stem layer (3x3/2 conv of a 3-channel image, bias, GELU) against the autocast
    arithmetic written in PyTorch: bf16 inputs and weights, fp32 sums, bf16 convolution output,
    fp32 bias and exact GELU, one rounding."""
    import torch.nn.functional as F

    from visionhope_b200.utils.bias_act import stem_conv

    g = torch.Generator(device=cuda).manual_seed(cout + H)
    x = torch.randn(3, 3, H, W, device=cuda, generator=g).contiguous(memory_format=torch.channels_last)
    conv = torch.nn.Conv2d(3, cout, 3, stride=2, padding=1).to(cuda)
    y = stem_conv(x, conv, act, out_dtype=ydt)
    assert y.dtype == ydt and y.is_contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        c = F.conv2d(x.to(torch.bfloat16).double(), conv.weight.to(torch.bfloat16).double(), None, 2, 1)
        c = c.to(torch.bfloat16).double() + conv.bias.double().view(1, -1, 1, 1)
        if act == "gelu":
            c = F.gelu(c)
    assert y.shape == c.shape
    tol = 1e-2 if ydt == torch.bfloat16 else 4e-3
    assert rel_err(y.double().cpu().numpy(), c.cpu().numpy()) < tol


@pytest.mark.parametrize("M,K,N", [(802816, 64, 32), (1000, 32, 32), (37, 64, 64), (517, 128, 256), (4099, 256, 128),
                                   (16, 32, 256)])
def test_rows_gemm(M, K, N, cuda):
    """Row GEMM of the 1x1 projections against F.linear with the same bf16 operands: fp32 sums
    in another order, so within a bf16 rounding; ragged row counts included."""
    import torch.nn.functional as F

    from visionhope_b200.utils.inference import rows_gemm

    g = torch.Generator(device=cuda).manual_seed(M + K + N)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    b = (torch.randn(N, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    y = rows_gemm(x, w, b.float())
    exp = F.linear(x.double(), w.double(), b.double())
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    assert rel_err(y.double().cpu().numpy(), exp.cpu().numpy()) < 4e-3
    y0 = rows_gemm(x, w, None)
    assert rel_err(y0.double().cpu().numpy(), (exp - b.double()).cpu().numpy()) < 4e-3


@pytest.mark.parametrize("M,K,N", [(802816, 64, 32), (200704, 128, 64), (1000, 32, 32), (37, 64, 64),
                                   (4099, 128, 32), (16, 32, 64)])
def test_ln_rows_gemm(M, K, N, cuda):
    """norm1 -> proj_in in one kernel against (a) the two kernels it replaces (LayerNorm
    writing bf16, then the row GEMM) and (b) an fp64 restatement of LayerNorm, bf16 rounding
    and F.linear.  The row statistics are summed in another order than the LayerNorm kernel's,
    so a normalized value can differ by one bf16 rounding: both within 4e-3 normwise."""
    import torch.nn.functional as F

    from visionhope_b200.utils.inference import ln_rows_gemm, rows_gemm
    from visionhope_b200.utils.layer_norm_cuda import layernorm_rows

    g = torch.Generator(device=cuda).manual_seed(3 * M + K + N)
    x = torch.randn(M, K, device=cuda, generator=g) * 2.0 + 0.5
    lw = 1.0 + 0.02 * torch.randn(K, device=cuda, generator=g)
    lb = 0.02 * torch.randn(K, device=cuda, generator=g)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    b = (torch.randn(N, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    eps = 1e-6
    y = ln_rows_gemm(x, lw, lb, eps, w, b.float())
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    two = rows_gemm(layernorm_rows(x, lw, lb, eps, out_dtype=torch.bfloat16), w, b.float())
    assert rel_err(y.double().cpu().numpy(), two.double().cpu().numpy()) < 4e-3
    n = F.layer_norm(x.double(), (K,), lw.double(), lb.double(), eps).to(torch.bfloat16).double()
    exp = F.linear(n, w.double(), b.double())
    assert rel_err(y.double().cpu().numpy(), exp.cpu().numpy()) < 4e-3
    y0 = ln_rows_gemm(x, lw, lb, eps, w, None)
    assert rel_err(y0.double().cpu().numpy(), (exp - b.double()).cpu().numpy()) < 4e-3


def test_ln_rows_gemm_rejects_shapes(cuda):
    from visionhope_b200.utils.inference import ln_rows_gemm

    x = torch.zeros(8, 256, device=cuda)
    ones, zeros = torch.ones(256, device=cuda), torch.zeros(256, device=cuda)
    with pytest.raises(RuntimeError):
        ln_rows_gemm(x, ones, zeros, 1e-6, torch.zeros(32, 256, device=cuda, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError):  # bf16 x: the kernel reads the fp32 residual stream
        ln_rows_gemm(x[:, :64].to(torch.bfloat16), ones[:64], zeros[:64], 1e-6,
                     torch.zeros(32, 64, device=cuda, dtype=torch.bfloat16))


def test_rows_gemm_rejects_shapes(cuda):
    from visionhope_b200.utils.inference import rows_gemm

    x = torch.zeros(8, 48, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        rows_gemm(x, torch.zeros(32, 48, device=cuda, dtype=torch.bfloat16))


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(128, 56, 56, 96), (128, 7, 7, 768)], ids=["128x56x56x96", "128x7x7x768"])
def test_grn_layernorm_config3_full_shapes(shape, dt, oracle, cuda):
    """The GRN/LN configuration at its stated shapes and batch (128), seed 2: LN gamma ~ N(1, 0.02),
    beta ~ N(0, 0.02); GRN gamma, beta ~ N(0, 0.02).  GRN (standalone and statistics-fed apply)
    and LayerNorm against the oracle, 1e-5 normwise (fp32 outputs)."""
    from visionhope_b200.utils.grn_cuda import grn_apply, grn_forward
    from visionhope_b200.utils.layer_norm_cuda import layernorm_rows

    B, H, W, C = shape
    gen = np.random.default_rng(2)
    x_nhwc = gen.normal(size=(B, H, W, C)).astype(np.float32)
    x = _dev(x_nhwc, cuda, DT[dt])
    xr = x.float().cpu().numpy()  # the values the kernels see
    lw, lb = gen.normal(1, 0.02, size=C), gen.normal(0, 0.02, size=C)
    gg, gb = gen.normal(0, 0.02, size=C), gen.normal(0, 0.02, size=C)

    y = layernorm_rows(x.reshape(-1, C), _dev(lw, cuda), _dev(lb, cuda), 1e-6)
    exp = oracle.layernorm_rows(xr.reshape(-1, C), lw, lb)
    assert rel_err(y.cpu().numpy(), exp) < 1e-5

    xc = x.permute(0, 3, 1, 2)  # channels-last logical NCHW
    exp = oracle.grn_nhwc(xr, gg, gb)
    g = grn_forward(xc, _dev(gg, cuda), _dev(gb, cuda), 1e-6)
    assert rel_err(g.permute(0, 2, 3, 1).cpu().numpy(), exp) < 1e-5
    sums = x.float().pow(2).sum(dim=(1, 2)).reshape(B, 1, C)
    ga = grn_apply(xc, sums, _dev(gg, cuda), _dev(gb, cuda), 1e-6)
    assert rel_err(ga.permute(0, 2, 3, 1).cpu().numpy(), exp) < 1e-5
