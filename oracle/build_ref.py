"""Compile the reference's own CUDA kernels into ``oracle/_ref/`` (test infrastructure only).

PSRben/VisionHOPE has no CPU implementation of SRNL, direction fusion or query
normalization (``models/srnl.py:113-114`` rejects CPU tensors), and ships no golden
vectors.  The strongest parity pin available is therefore the reference's own CUDA
extensions, run on a B200.  This recipe:

1. imports the reference package read-only from its checkout (``VHOPE_REFERENCE``; with a
   four-alias ``timm`` shim, because timm is not installed) so that the reference
   renders its own templated sources exactly as it does at run time
   (``models/srnl_core/fused.py:51-64``, ``chunk.py:89-105``, ``lines.py:59-70``,
   ``utils/query_normalization.py:28-33``, ``utils/direction_fusion.py:39-41``);
2. compiles those rendered strings with ``torch.utils.cpp_extension.load_inline``
   for sm_100a into ``oracle/_ref/<name>/`` (git-ignored; the built ``.so`` files
   travel to the GPU box, the sources never enter the repository).

The reference's own JIT loaders are not called; only the build flags it uses
(``-O3 --use_fast_math``) are mirrored, plus an explicit ``-gencode`` for sm_100a.

``stage_python`` also copies the reference's Python package, unmodified (its ``models/``
and ``utils/`` trees with the kernel sources they read at import, ``inference/prepare.py``),
into ``oracle/_ref/pyref/visionhope/`` (git-ignored, like the built kernels), so that tests
on the GPU box, where no reference checkout exists, can run the reference's own modules:
with its own kernels (``oracle/refmodel.py``, mode "native") and over this repository's
drop-in modules (mode "dropin").
Nothing in the product imports this module or its outputs.
"""
from __future__ import annotations

import os
import sys
import tempfile
import types
from pathlib import Path

# The reference checkout: the VHOPE_REFERENCE environment variable (no default location).
REF_ROOT = Path(os.environ["VHOPE_REFERENCE"]) if os.environ.get("VHOPE_REFERENCE") else None
OUT_DIR = Path(__file__).resolve().parent / "_ref"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _install_reference():
    base = tempfile.mkdtemp(prefix="vhref_")
    os.symlink(REF_ROOT, os.path.join(base, "visionhope"))
    sys.path.insert(0, base)
    install_timm_shim()


def install_timm_shim():
    """timm is not installed; the reference uses only these five names from it
    (trunc_normal_, DropPath, register_model and the ImageNet mean/std)."""
    import torch

    if "timm" not in sys.modules:
        timm = types.ModuleType("timm")
        models = types.ModuleType("timm.models")
        layers = types.ModuleType("timm.models.layers")
        registry = types.ModuleType("timm.models.registry")
        data = types.ModuleType("timm.data")
        layers.trunc_normal_ = lambda t, mean=0.0, std=1.0, a=-2.0, b=2.0: torch.nn.init.trunc_normal_(
            t, mean, std, a, b)

        class DropPath(torch.nn.Module):
            def __init__(self, p=0.0):
                super().__init__()
                self.drop_prob = p

            def forward(self, x):
                return x

        layers.DropPath = DropPath
        registry.register_model = lambda f: f
        data.IMAGENET_DEFAULT_MEAN = (0.485, 0.456, 0.406)
        data.IMAGENET_DEFAULT_STD = (0.229, 0.224, 0.225)
        timm.models, models.layers, models.registry, timm.data = models, layers, registry, data
        for name, mod in (("timm", timm), ("timm.models", models), ("timm.models.layers", layers),
                          ("timm.models.registry", registry), ("timm.data", data)):
            sys.modules[name] = mod


def _targets():
    """(extension name, cpp source, cuda source, exported functions) for every kernel we pin."""
    import torch
    import visionhope.models.srnl_core.chunk as chunk
    import visionhope.models.srnl_core.fused as fused
    import visionhope.models.srnl_core.lines as lines
    import visionhope.utils.direction_fusion as dirfuse
    import visionhope.utils.query_normalization as qnorm

    fused_fns = ["srnl_line_forward_seq_noatomic", "srnl_sequence_forward"]
    chunk_fns = ["srnl_forward", "srnl_forward_qraw", "srnl_backward", "srnl_backward_qraw"]
    line_fns = ["srnl_forward_qraw_large", "srnl_backward_qraw_large", "srnl_forward_qraw_varline",
                "srnl_backward_qraw_varline"]
    qnorm_fns = ["visionhope_qnorm_forward", "visionhope_qnorm_backward"]
    dirfuse_fns = ["visionhope_postprocess_scale_forward", "visionhope_postprocess_scale_backward"]
    base_chunk = chunk.cuda_helper_source
    return [
        ("vhref_fused_bf16", fused.cpp_source, fused.cuda_source, fused_fns),
        ("vhref_fused_fp32", fused.cpp_source, fused.cuda_source_fp32, fused_fns),
        ("vhref_chunk_bf16", chunk.cpp_source, chunk.cuda_source, chunk_fns),
        ("vhref_chunk_fp32", chunk.cpp_source, chunk.cuda_source_fp32, chunk_fns),
        ("vhref_lines_bf16", lines.cpp_source,
         base_chunk + lines.large_cuda_source + lines.varline_cuda_source, line_fns),
        ("vhref_lines_fp32", lines.cpp_source,
         base_chunk + lines.large_cuda_source_fp32 + lines.varline_cuda_source_fp32, line_fns),
        ("vhref_qnorm_bf16", qnorm.cpp_source, qnorm.cuda_source, qnorm_fns),
        ("vhref_qnorm_fp32", qnorm.cpp_source, qnorm.cuda_source_fp32, qnorm_fns),
        ("vhref_dirfuse_bf16", dirfuse.cpp_source, dirfuse.cuda_source, dirfuse_fns),
        ("vhref_dirfuse_fp32", dirfuse.cpp_source, dirfuse.cuda_source_fp32, dirfuse_fns),
    ]


def _grn_target():
    src = REF_ROOT / "utils" / "csrc"
    return "vhref_grn", [str(src / "grn.cpp"), str(src / "grn_cuda.cu")]


def _names():
    return [t[0] for t in _targets()] + [_grn_target()[0]]


def build_parallel(workers=None):
    """Build every reference extension, several at a time in spawned processes (each one is a
    separate nvcc job of a few minutes; built ones are up to date and return at once)."""
    import concurrent.futures as cf
    import multiprocessing as mp

    if REF_ROOT is None or not REF_ROOT.is_dir():
        raise FileNotFoundError(f"reference tree not found (VHOPE_REFERENCE={REF_ROOT})")
    _install_reference()
    names = _names()
    workers = workers or max(1, min(len(names), (os.cpu_count() or 2) // 2))
    built = []
    with cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")) as ex:
        for res in ex.map(build, [[n] for n in names]):
            built += res
    return built


def build(only=None):
    if REF_ROOT is None or not REF_ROOT.is_dir():
        raise FileNotFoundError(f"reference tree not found (VHOPE_REFERENCE={REF_ROOT})")
    _install_reference()
    from torch.utils.cpp_extension import load, load_inline

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    flags = ["-O3", "--use_fast_math", *GENCODE]
    built = []
    def fresh_dir(name):
        # A build killed half-way leaves torch's `lock` file behind, and the next build of the
        # same extension would wait on it for ever; this script builds each extension in one
        # process only, so a lock found here is always such a leftover.
        d = OUT_DIR / name
        d.mkdir(parents=True, exist_ok=True)
        (d / "lock").unlink(missing_ok=True)
        return d

    for name, cpp, cuda, fns in _targets():
        if only and name not in only:
            continue
        build_dir = fresh_dir(name)
        load_inline(name=name, cpp_sources=cpp, cuda_sources=cuda, functions=fns,
                    extra_cuda_cflags=flags, build_directory=str(build_dir), verbose=False)
        built.append(name)
    name, sources = _grn_target()
    if not only or name in only:
        build_dir = fresh_dir(name)
        load(name=name, sources=sources, extra_cuda_cflags=["-O3", *GENCODE], extra_cflags=["-O3"],
             build_directory=str(build_dir), verbose=False)
        built.append(name)
    return built


PYREF_DIR = OUT_DIR / "pyref"
_STAGED = ("__init__.py", "models", "utils", "inference/__init__.py", "inference/prepare.py",
           "tasks/__init__.py", "tasks/backbone.py", "tools/__init__.py", "tools/checkpoint.py")


def stage_python():
    """Copy the reference's Python package (unmodified) into ``oracle/_ref/pyref/visionhope``."""
    import shutil

    if REF_ROOT is None or not REF_ROOT.is_dir():
        raise FileNotFoundError(f"reference tree not found (VHOPE_REFERENCE={REF_ROOT})")
    dst = PYREF_DIR / "visionhope"
    if dst.exists():
        shutil.rmtree(dst)
    keep = shutil.ignore_patterns("__pycache__", "*.pyc", "*.md", "*.png")
    for rel in _STAGED:
        src = REF_ROOT / rel
        out = dst / rel
        out.parent.mkdir(parents=True, exist_ok=True)
        if src.is_dir():
            shutil.copytree(src, out, ignore=keep)
        else:
            shutil.copy2(src, out)
    return dst


_loaded = {}


def load_built(name):
    """Import a previously built reference extension from ``oracle/_ref/<name>/`` (once per
    process; an extension module cannot be initialised twice)."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch)

    if name in _loaded:
        return _loaded[name]
    path = OUT_DIR / name / f"{name}.so"
    if not path.is_file():
        raise FileNotFoundError(f"reference extension {name} not built at {path}")
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    _loaded[name] = module
    return module


if __name__ == "__main__":
    print("staged:", stage_python())
    print("built:", build(sys.argv[1:]) if sys.argv[1:] else build_parallel())
