"""The reference's own VisionHOPE modules, imported for parity tests (TEST INFRASTRUCTURE).

Imports the reference package staged unmodified by ``oracle/build_ref.py:stage_python`` into
``oracle/_ref/pyref/visionhope`` (git-ignored; it travels to the GPU box with the built
reference kernels).  Nothing in the product imports this module.  Two modes:

``"native"``  the reference exactly as it runs: its modules on its own CUDA kernels.  The
             kernels are the ones ``build_ref.build`` compiled from the reference's sources
             for sm_100a; the reference's JIT loaders (``models/srnl_core/fused.py:67-93``,
             ``chunk.py:108-165``, ``lines.py:79-180``, ``utils/query_normalization.py:36-54``,
             ``utils/direction_fusion.py:46-84``, ``utils/grn_cuda.py:19-30``) are pointed at
             those builds instead of compiling at first use.
``"dropin"``  the reference's modules unchanged (``models/*.py``, ``inference/prepare.py``)
             with the modules this repository replaces -- ``models/srnl_core`` and
             ``utils/{direction_fusion,grn,grn_cuda,layer_norm_cuda,query_normalization,residual}`` --
             bound to ``visionhope_b200``'s, as a user integrating the drop-in would
             (option A).

Only one mode is imported at a time: ``load`` drops every ``visionhope.*`` module of the
previous mode first (``visionhope_b200`` modules stay).
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path
from types import SimpleNamespace

from oracle import build_ref

PYREF = build_ref.PYREF_DIR

# reference module -> the module of this repository that replaces it
DROPIN = {
    "visionhope.models.srnl_core": "visionhope_b200.srnl_core",
    "visionhope.models.srnl_core.chunk": "visionhope_b200.srnl_core.chunk",
    "visionhope.models.srnl_core.lines": "visionhope_b200.srnl_core.lines",
    "visionhope.models.srnl_core.fused": "visionhope_b200.srnl_core.fused",
    "visionhope.utils.direction_fusion": "visionhope_b200.utils.direction_fusion",
    "visionhope.utils.grn": "visionhope_b200.utils.grn",
    "visionhope.utils.grn_cuda": "visionhope_b200.utils.grn_cuda",
    "visionhope.utils.layer_norm_cuda": "visionhope_b200.utils.layer_norm_cuda",
    "visionhope.utils.query_normalization": "visionhope_b200.utils.query_normalization",
    "visionhope.utils.residual": "visionhope_b200.utils.residual",
}


def available() -> bool:
    return (PYREF / "visionhope" / "models" / "operator.py").is_file()


def kernels_available() -> bool:
    return all((build_ref.OUT_DIR / n / f"{n}.so").is_file()
               for n in ("vhref_fused_bf16", "vhref_chunk_fp32", "vhref_qnorm_bf16", "vhref_dirfuse_fp32"))


def _purge():
    for name in list(sys.modules):
        if name == "visionhope" or name.startswith("visionhope."):
            del sys.modules[name]


def _by_dtype(prefix):
    import torch

    cache = {}

    def loader(io_dtype=torch.bfloat16, *_):
        tag = {torch.bfloat16: "bf16", torch.float32: "fp32"}.get(io_dtype)
        if tag is None:
            raise TypeError(f"no reference build of {prefix} for {io_dtype}")
        if tag not in cache:
            cache[tag] = build_ref.load_built(f"{prefix}_{tag}")
        return cache[tag]
    return loader


def _patch_native():
    import visionhope.models.srnl_core.chunk as chunk
    import visionhope.models.srnl_core.fused as fused
    import visionhope.models.srnl_core.lines as lines
    import visionhope.utils.direction_fusion as dirfuse
    import visionhope.utils.grn_cuda as grn_cuda
    import visionhope.utils.query_normalization as qnorm

    fused.load_fused_cuda = _by_dtype("vhref_fused")
    chunk.load_cuda = _by_dtype("vhref_chunk")
    lines.load_cuda = _by_dtype("vhref_lines")
    qnorm.load_qnorm_cuda = _by_dtype("vhref_qnorm")
    dirfuse.load_postprocess_cuda = _by_dtype("vhref_dirfuse")
    grn_mod = []

    def grn_loader():
        if not grn_mod:
            grn_mod.append(build_ref.load_built("vhref_grn"))
        return grn_mod[0]
    grn_cuda._load_cuda_extension = grn_loader

    # The Triton LayerNorm and residual kernels size their rows from
    # triton.runtime.driver.utils.get_device_properties()["max_shared_mem"]
    # (utils/layer_norm_cuda.py:18-22, utils/residual.py:18-21), which the installed Triton no
    # longer provides; the same number (the opt-in shared memory per block) comes from torch.
    import visionhope.utils.layer_norm_cuda as ln_mod
    import visionhope.utils.residual as res_mod

    def row_capacity(device):
        import torch
        return torch.cuda.get_device_properties(device).shared_memory_per_block_optin // (8 * 4)
    ln_mod._row_capacity = row_capacity
    res_mod._row_capacity = row_capacity


def load(mode: str) -> SimpleNamespace:
    """Import the reference package in ``mode`` ("native" or "dropin"); returns its
    ``models`` package, ``prepare_for_inference`` and ``create_model``."""
    if mode not in ("native", "dropin"):
        raise ValueError(mode)
    if not available():
        raise FileNotFoundError(f"reference package not staged at {PYREF}")
    _purge()
    build_ref.install_timm_shim()
    if str(PYREF) not in sys.path:
        sys.path.insert(0, str(PYREF))
    if mode == "dropin":
        for ref_name, ours in DROPIN.items():
            sys.modules[ref_name] = importlib.import_module(ours)
    models = importlib.import_module("visionhope.models")
    prepare = importlib.import_module("visionhope.inference.prepare")
    if mode == "native":
        _patch_native()
    return SimpleNamespace(mode=mode, models=models, create_model=models.create_model,
                           prepare_for_inference=prepare.prepare_for_inference,
                           SRNL=models.SRNL, VisionHOPEOperator=models.VisionHOPEOperator)
