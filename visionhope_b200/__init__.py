"""visionhope_b200: VisionHOPE's inference hot path on NVIDIA B200 (sm_100a).

The SRNL five-memory recurrence run as four directional chunked scans, spatial
restoration and channel-wise direction fusion, query normalization, GRN and LayerNorm,
as hand-written CUDA in ``libvhope.so`` (C ABI: ``include/vhope.h``), behind host-side
mirrors of the reference's Python interfaces:

    visionhope_b200.srnl_core      <- models/srnl_core
    visionhope_b200.srnl.SRNL      <- models/srnl.py
    visionhope_b200.operator       <- models/operator.py
    visionhope_b200.utils.*        <- utils/{direction_fusion,grn,grn_cuda,layer_norm_cuda,
                                             query_normalization,cuda}.py
"""
from ._lib import load as load_library, version  # noqa: F401

__version__ = "0.1.0"
