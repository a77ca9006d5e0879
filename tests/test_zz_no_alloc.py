"""GRN without device allocation, through the C ABI.

vh_grn_fwd_noalloc exists for callers that cannot allocate device memory while they run
(plugin/serving hosts that pass an op only its inputs and outputs, deployments with a fixed
device-memory budget).  It keeps its partial sums in an array built into the library, so this
test checks that calls in a row -- each on different data, so the array holds the previous
call's leftovers -- each match the workspace entry point vh_grn_fwd within the GRN tolerance
used elsewhere in these tests (1e-5 normwise), that the first one also matches the CPU oracle,
and that an oversized call is refused.  The third shape (256 x 7 x 7 x 2048, batch * channels
= 524,288) is close enough to the array's limit that the entry point runs 2 pixel slices per
image where vh_grn_fwd runs 3, so the clamped split count and its slicing are exercised.
The file sorts last so a stop-at-first-failure run has already run everything else.
"""
import ctypes

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _lib():
    from visionhope_b200 import _lib as L

    lib = L.load()
    lib.vh_grn_fwd_noalloc.restype = ctypes.c_int32
    lib.vh_grn_fwd_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_void_p]
    return L, lib


def _with_workspace(L, lib, x, gamma, beta, stream):
    B, H, W, C = x.shape
    y = torch.empty_like(x, dtype=torch.float32)
    gx = torch.empty(B, C, device=x.device)
    inv = torch.empty(B, device=x.device)
    nbytes = lib.vh_grn_workspace_bytes(B, H, W, C)
    ws = torch.empty((nbytes + 3) // 4, device=x.device)
    rc = lib.vh_grn_fwd(x.data_ptr(), L.dtype_code(x.dtype), gamma.data_ptr(), beta.data_ptr(), 1e-6,
                        y.data_ptr(), 0, gx.data_ptr(), inv.data_ptr(), ws.data_ptr(), ws.numel() * 4,
                        B, H, W, C, stream)
    assert rc == 0, lib.vh_last_error()
    return y, gx, inv


def _no_alloc(L, lib, x, gamma, beta, stream):
    B, H, W, C = x.shape
    y = torch.empty_like(x, dtype=torch.float32)
    gx = torch.empty(B, C, device=x.device)
    inv = torch.empty(B, device=x.device)
    rc = lib.vh_grn_fwd_noalloc(x.data_ptr(), L.dtype_code(x.dtype), gamma.data_ptr(), beta.data_ptr(),
                                1e-6, y.data_ptr(), gx.data_ptr(), inv.data_ptr(), B, H, W, C, stream)
    assert rc == 0, lib.vh_last_error()
    return y, gx, inv


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_no_alloc_grn_matches_workspace_grn_twice(dtype, oracle):
    assert torch.cuda.is_available()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    L, lib = _lib()
    L.ensure_device(torch.empty(1, device=dev))
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(17)
    # each call after the first: different data and shape; the last one near the array's limit
    shapes = [(4, 14, 14, 96), (3, 7, 7, 768), (256, 7, 7, 2048)]
    for i, (B, H, W, C) in enumerate(shapes):
        x = torch.randn(B, H, W, C, device=dev, generator=g).to(dtype)
        gamma = torch.randn(C, device=dev, generator=g) * 0.02
        beta = torch.randn(C, device=dev, generator=g) * 0.02
        ref = _with_workspace(L, lib, x, gamma, beta, stream)
        got = _no_alloc(L, lib, x, gamma, beta, stream)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.isfinite(a).all()
            assert rel_err(a, b) < 1e-5
        if i == 0:
            exp = oracle.grn_nhwc(x.float().cpu().numpy(), gamma.cpu().numpy(), beta.cpu().numpy())
            assert rel_err(got[0], exp) < 1e-5
        if i == 1:
            lib.vh_grn_noalloc_reset()  # the next call looks the array's address up again


def test_no_alloc_split_count_is_clamped():
    """At 256 x 7 x 7 x 2048 the workspace entry point runs 3 slices per image, more than the
    built-in array holds for that batch * channels, so the no-alloc call must run fewer."""
    _, lib = _lib()
    lib.vh_grn_workspace_bytes.restype = ctypes.c_int64
    slices = lib.vh_grn_workspace_bytes(256, 7, 7, 2048) // (4 * 256 * 2048)
    assert slices == 3 and slices * 256 * 2048 > (1 << 20)


def test_no_alloc_grn_rejects_oversized_batch():
    dev = torch.device("cuda:0")
    L, lib = _lib()
    L.ensure_device(torch.empty(1, device=dev))
    x = torch.empty(8, 1, 1, 262144 // 2 * 2, device=dev)  # batch * channels = 2,097,152 > 1,048,576
    g = torch.zeros(x.shape[-1], device=dev)
    y = torch.empty_like(x)
    rc = lib.vh_grn_fwd_noalloc(x.data_ptr(), 0, g.data_ptr(), g.data_ptr(), 1e-6, y.data_ptr(), None, None,
                                8, 1, 1, x.shape[-1], torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -6
    assert b"exceeds the built-in scratch" in lib.vh_last_error()
