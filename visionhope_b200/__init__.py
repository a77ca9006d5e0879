"""visionhope_b200: VisionHOPE's inference hot path on NVIDIA B200 (sm_100a).

The SRNL five-memory recurrence run as four directional chunked scans, spatial
restoration and channel-wise direction fusion, query normalization, GRN and LayerNorm,
as hand-written CUDA in ``libvhope.so`` (C ABI: ``include/vhope.h``), behind drop-in
replacements of the reference modules that own its kernels:

    visionhope_b200.srnl_core      <- models/srnl_core
    visionhope_b200.utils.*        <- utils/{direction_fusion,grn,grn_cuda,layer_norm_cuda,
                                             query_normalization}.py

The reference's own ``models/srnl.py``, ``models/operator.py`` and ``models/block.py`` run
unchanged on top of them.  ``visionhope_b200.backbone`` (with ``mixer``) is a separate
caller harness that drives the kernels end to end for the whole-model benchmark.
"""
from ._lib import load as load_library, version  # noqa: F401

__version__ = "0.1.0"
