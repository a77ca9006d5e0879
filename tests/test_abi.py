"""C-ABI checks that need no GPU: the library loads, exports every symbol declared in
include/vhope.h, and rejects invalid arguments before any CUDA call (status + message)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "vhope.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|void|const char\*)\s+(vh_\w+)\s*\(", text, re.M)))


def test_header_declares_the_entry_points():
    names = declared_symbols()
    for want in ("vh_srnl_spatial_fwd", "vh_srnl_sequence_fwd", "vh_qnorm_fwd", "vh_dirfuse_fwd",
                 "vh_grn_fwd", "vh_grn_workspace_bytes", "vh_layernorm_fwd", "vh_init",
                 "vh_last_error", "vh_last_launch_count", "vh_version"):
        assert want in names


def test_library_exports_every_declared_symbol():
    from visionhope_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert "sm_100a" in _lib.version()


def test_struct_layouts_match_header_sizes():
    from visionhope_b200 import _lib

    # 6 x 4-byte fields; 5 pointers + int (padded); see include/vhope.h
    assert ctypes.sizeof(_lib.VhConsts) == 24
    assert ctypes.sizeof(_lib.VhMemories) == 48
    assert ctypes.sizeof(_lib.VhSequenceArgs) == 48 + 3 * 8 + 8 * 4 + 4 * 4 + 24 + 0


def _c_layout(struct, fields):
    """sizeof and offsetof of `fields` of a header struct, compiled with the host C compiler."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    body = "".join(f'printf("%zu\\n", offsetof({struct}, {f}));\n' for f in fields)
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include \"vhope.h\"\n"
           f"int main(void) {{ printf(\"%zu\\n\", sizeof({struct}));\n{body} return 0; }}\n")
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "layout.c", Path(d) / "layout"
        c.write_text(src)
        subprocess.run([cc, "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
        vals = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                               text=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("struct,cls", [("vh_srnl_spatial_args", "VhSpatialArgs"),
                                        ("vh_srnl_sequence_args", "VhSequenceArgs"),
                                        ("vh_srnl_consts", "VhConsts"),
                                        ("vh_srnl_memories", "VhMemories"),
                                        ("vh_dwconv_args", "VhDwconvArgs")])
def test_ctypes_mirrors_match_the_header(struct, cls):
    """Every field of the ctypes mirrors sits at the offset the C compiler gives it."""
    from visionhope_b200 import _lib

    py = getattr(_lib, cls)
    names = [f[0] for f in py._fields_]
    size, offsets = _c_layout(struct, names)
    assert ctypes.sizeof(py) == size
    assert [getattr(py, n).offset for n in names] == offsets


def _err(lib):
    return lib.vh_last_error().decode()


def test_null_arguments_are_rejected_without_a_gpu():
    from visionhope_b200 import _lib

    lib = _lib.load()
    assert lib.vh_srnl_spatial_fwd(None, None) == -1
    assert "null" in _err(lib)
    args = _lib.VhSpatialArgs()
    assert lib.vh_srnl_spatial_fwd(ctypes.byref(args), None) == -1
    seq = _lib.VhSequenceArgs()
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq), None) == -1
    assert lib.vh_qnorm_fwd(None, 1, None, None, 1, 4, 1, 1, 16, None) == -1
    assert lib.vh_dirfuse_fwd(None, None, 1, None, 0, None, None, 0, 1, 1, 1, 1, 16, None) == -1
    assert lib.vh_layernorm_fwd(None, 0, None, None, 1e-6, None, 0, None, None, 1, 4, None) == -1


def _fake(n=1 << 12):
    """A host buffer used only as a non-null, aligned address (validation never dereferences)."""
    buf = (ctypes.c_float * n)()
    return ctypes.addressof(buf), buf


@pytest.mark.parametrize("head_dim,code", [(12, -4), (0, -4), (128, -4)])
def test_bad_head_dim(head_dim, code):
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    seq = _lib.VhSequenceArgs(_lib.VhMemories(p, p, p, p, p, 0), p, p, p, 0, 0, 0, 1, 1, 1, 8,
                              head_dim, (_lib.c_int32 * 4)(4, 4, 4, 4), _lib.consts(0.025, 0, 2.2, 0.999, 0.999999))
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq), None) == code
    assert "head_dim" in _err(lib)


def test_sequence_validation_messages():
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    k = _lib.consts(0.025, 0, 2.2, 0.999, 0.999999)

    def seq(**kw):
        base = dict(x_dtype=0, q_dtype=0, q_mode=0, batch=1, dirs=1, heads=1, length=8, head_dim=16,
                    chunk=(4, 4, 4, 4))
        base.update(kw)
        return _lib.VhSequenceArgs(_lib.VhMemories(p, p, p, p, p, 0), p, p, p, base["x_dtype"],
                                   base["q_dtype"], base["q_mode"], base["batch"], base["dirs"],
                                   base["heads"], base["length"], base["head_dim"],
                                   (_lib.c_int32 * 4)(*base["chunk"]), k)

    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(dirs=3)), None) == -2
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(batch=0)), None) == -2
    assert "nonempty" in _err(lib)
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(chunk=(0, 4, 4, 4))), None) == -2
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(x_dtype=1, q_dtype=0)), None) == -3
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(q_mode=1, q_dtype=1, x_dtype=1)), None) == -3
    assert lib.vh_srnl_sequence_fwd(ctypes.byref(seq(x_dtype=7, q_dtype=7)), None) == -3


def test_spatial_misalignment_is_rejected():
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    k = _lib.consts(0.025, 0, 2.2, 0.999, 0.999999)
    C = 32
    args = _lib.VhSpatialArgs(_lib.VhMemories(p, p, p, p, p, 0), p + 2, p, 4 * 16 * C, 16 * C, C, 16,
                              4 * 16 * C, 16 * C, C, 16, 1, 0, p, 0, p, p, 16 * C, 1, 4, 4, 2, 16, k)
    assert lib.vh_srnl_spatial_fwd(ctypes.byref(args), None) == -5
    assert "aligned" in _err(lib)


def test_grn_workspace_query():
    from visionhope_b200 import _lib

    lib = _lib.load()
    assert lib.vh_grn_workspace_bytes(128, 56, 56, 96) > 0
    assert lib.vh_grn_workspace_bytes(0, 56, 56, 96) == 0


def test_harness_entry_points_validate_without_a_gpu():
    """The harness kernels' entry points reject bad shapes, dtypes and pointers with a status
    and a message before any CUDA call."""
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    # row GEMM: unsupported feature counts, empty input, misaligned x
    assert lib.vh_rows_gemm_fwd(p, p, p, p, 16, 48, 32, None) == -2
    assert "in/out features" in _err(lib)
    assert lib.vh_rows_gemm_fwd(p, p, p, p, 0, 64, 32, None) == -2
    assert lib.vh_rows_gemm_fwd(p + 4, p, p, p, 16, 64, 32, None) == -5
    assert lib.vh_rows_gemm_fwd(None, p, p, p, 16, 64, 32, None) == -1
    # LayerNorm + row GEMM: feature counts, empty input, eps, misaligned x, null pointers
    assert lib.vh_ln_rows_gemm_fwd(p, p, p, 1e-6, p, p, p, 16, 256, 32, None) == -2
    assert "in_features" in _err(lib)
    assert lib.vh_ln_rows_gemm_fwd(p, p, p, 1e-6, p, p, p, 16, 64, 128, None) == -2
    assert lib.vh_ln_rows_gemm_fwd(p, p, p, 1e-6, p, p, p, 0, 64, 32, None) == -2
    assert lib.vh_ln_rows_gemm_fwd(p, p, p, -1.0, p, p, p, 16, 64, 32, None) == -1
    assert lib.vh_ln_rows_gemm_fwd(p + 4, p, p, 1e-6, p, p, p, 16, 64, 32, None) == -5
    assert lib.vh_ln_rows_gemm_fwd(p, None, p, 1e-6, p, p, p, 16, 64, 32, None) == -1
    # stem convolution: output channels, activation, dtype
    assert lib.vh_stem_conv_fwd(p, p, p, p, 1, 2, 32, 32, 40, 1, None) == -2
    assert "out_channels" in _err(lib)
    assert lib.vh_stem_conv_fwd(p, p, p, p, 1, 2, 32, 32, 32, 7, None) == -1
    assert lib.vh_stem_conv_fwd(p, p, p, p, 2, 2, 32, 32, 32, 1, None) == -3
    # add + cast: element count and dtype
    assert lib.vh_add_cast_fwd(p, 0, p, 1, p, 1, 12, None) == -2
    assert lib.vh_add_cast_fwd(p, 2, p, 1, p, 1, 16, None) == -3
    # statistics-fed GRN: channel count
    assert lib.vh_grn_apply_fwd(p, 1, p, 1, p, p, 1e-6, p, p, 1, 2, 4, 4, 12, None) == -2
    assert "channels" in _err(lib)
    assert lib.vh_grn_apply_fwd(p, 1, p, 1, p, p, 1e-6, p, p, 1, 2, 4, 4, 4096, None) == -2


def test_dwconv_gate_pos_validates_without_a_gpu():
    """The fused local-features + position mode rejects missing operands, other dtypes, other
    kernel sizes and images that a CTA does not hold whole, before any CUDA call."""
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()

    def args(**kw):
        a = dict(x=p, gate=p, weight=p, bias=p, y=p + 4096, dtype=1, mode=5, ksize=7, batch=2, height=14,
                 width=14, channels=32, gate_dtype=0, sumsq=None, pos_weight=p, pos_bias=p, pos_y=p + 8192,
                 pos_ksize=5)
        a.update(kw)
        return _lib.VhDwconvArgs(**a)

    assert lib.vh_dwconv_fwd(ctypes.byref(args(pos_y=None)), None) == -1
    assert "pos_y" in _err(lib)
    assert lib.vh_dwconv_fwd(ctypes.byref(args(dtype=0)), None) == -3
    assert lib.vh_dwconv_fwd(ctypes.byref(args(pos_ksize=3)), None) == -2
    assert lib.vh_dwconv_fwd(ctypes.byref(args(height=56, width=56)), None) == -2
    assert "14 x 14 or 7 x 7" in _err(lib)
    assert lib.vh_dwconv_fwd(ctypes.byref(args(pos_y=p)), None) == -1  # aliases x
    assert lib.vh_dwconv_fwd(ctypes.byref(args(mode=6)), None) == -1


def test_dwconv_tile_count_query():
    from visionhope_b200 import _lib

    lib = _lib.load()
    assert lib.vh_dwconv_tiles(56, 56) == 16   # 14 x 14 tiles
    assert lib.vh_dwconv_tiles(14, 14) == 1
    assert lib.vh_dwconv_tiles(7, 7) == 1      # whole images, four per CTA
    assert lib.vh_dwconv_tiles(32, 32) == 4    # 16 x 16 tiles
    assert lib.vh_dwconv_tiles(0, 5) == 0


def _bwd_args(lib_mod, p, **kw):
    base = dict(x_dtype=0, q_dtype=0, q_mode=0, batch=2, dirs=4, heads=2, length=100, head_dim=16,
                chunk=(100, 100, 100, 100))
    base.update(kw)
    k = lib_mod.consts(0.025, 0, 2.2, 0.999, 0.999999)
    return lib_mod.VhSequenceBwdArgs(lib_mod.VhMemories(p, p, p, p, p, 0), p, p, base["x_dtype"], base["q_dtype"],
                                     base["q_mode"], p, p, p, p, p, p, p, p, base["batch"], base["dirs"],
                                     base["heads"], base["length"], base["head_dim"],
                                     (lib_mod.c_int32 * 4)(*base["chunk"]), k)


def test_sequence_backward_validation_and_workspace(monkeypatch):
    """vh_srnl_sequence_bwd's host checks (no GPU): chunks past 64 tokens are taken for head_dim
    16 only; the workspace query grows with the kept gain history, which
    VHOPE_SRNL_BWD_HISTORY_BYTES=0 turns off; a short workspace is refused before any launch."""
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    a8 = _bwd_args(_lib, p, head_dim=8)
    assert lib.vh_srnl_sequence_bwd(ctypes.byref(a8), p, 1 << 40, None) == -6
    assert "MAX_CHUNK" in _err(lib)
    a16 = _bwd_args(_lib, p)
    full = lib.vh_srnl_sequence_bwd_workspace_bytes(ctypes.byref(a16))
    chains, n, Lc = 2 * 4 * 2, 1, 100
    # states + full history + dS + chunk-end gains (floats)
    assert full == 4 * chains * (n * 800 + n * Lc * 256 + 800 + n * 256)
    monkeypatch.setenv("VHOPE_SRNL_BWD_HISTORY_BYTES", "0")
    small = lib.vh_srnl_sequence_bwd_workspace_bytes(ctypes.byref(a16))
    assert small == 4 * chains * (n * 800 + Lc * 256 + 800)
    assert lib.vh_srnl_sequence_bwd(ctypes.byref(a16), p, small - 4, None) == -1
    assert "workspace too small" in _err(lib)


def test_residual_and_norm_backward_validation():
    from visionhope_b200 import _lib

    lib = _lib.load()
    p, keep = _fake()
    assert lib.vh_residual_add_fwd(p, 0, p, 9, p, p, p, 2, 4, 8, None) == -3
    assert lib.vh_residual_add_fwd(p, 0, p, 0, p, p, p, 0, 4, 8, None) == -2
    assert lib.vh_residual_add_fwd(None, 0, p, 0, p, p, p, 2, 4, 8, None) == -1
    need = lib.vh_residual_add_bwd_workspace_bytes(2 * 4, 8)
    assert need == 4 * 8  # one partial row for 8 rows
    assert lib.vh_residual_add_bwd(p, p, 0, p, p, p, p, p, need - 4, 2, 4, 8, None) == -1
    assert "workspace too small" in _err(lib)
    assert lib.vh_layernorm_bwd_workspace_bytes(1000, 96) == 4 * 2 * 96 * (4 + 1)
    assert lib.vh_layernorm_bwd(p, p, 0, p, p, p, p, p, p, p, 16, 1000, 96, None) == -1
