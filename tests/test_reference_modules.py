"""CPU checks of the drop-in boundary with the reference's own modules (``oracle/refmodel.py``):
the reference's modules import over this repository's replacements, the replacements keep the
names the reference imports, and the harness backbone loads a reference state_dict strictly."""
import pytest
import torch

from tests.conftest import reference


def test_dropin_binds_this_repository_modules():
    import importlib

    ref = reference("dropin")
    from oracle.refmodel import DROPIN

    for ref_name, ours in DROPIN.items():
        assert importlib.import_module(ref_name) is importlib.import_module(ours)
    import visionhope.models.srnl as srnl

    assert srnl.srnl_raw_query.__module__ == "visionhope_b200.srnl_core.chunk"
    assert ref.SRNL.__module__ == "visionhope.models.srnl"


def test_reference_names_resolve_on_the_dropin():
    """Every name models/srnl.py, models/operator.py, models/layers.py and models/block.py import
    from the replaced modules exists in this repository's modules."""
    reference("dropin")
    import visionhope.models.srnl_core as core
    import visionhope.models.srnl_core.chunk as chunk
    import visionhope.models.srnl_core.fused as fused
    import visionhope.utils.direction_fusion as dirfuse
    import visionhope.utils.grn as grn
    import visionhope.utils.layer_norm_cuda as ln
    import visionhope.utils.query_normalization as qn

    for mod, names in ((core, ["MAX_CHUNK", "SUPPORTED_HEAD_DIMS", "srnl_long_chunk", "srnl_normalized_query",
                               "srnl_raw_query", "srnl_variable_lines"]),
                       (chunk, ["can_fuse_raw_query"]),
                       (fused, ["srnl_sequence_inference", "load_fused_cuda"]),
                       (dirfuse, ["can_fuse_scale_postprocess", "visionhope_postprocess_scale"]),
                       (grn, ["GlobalResponseNorm", "global_response_norm", "grn_reference"]),
                       (ln, ["can_fuse_layernorm2d", "visionhope_layernorm2d"]),
                       (qn, ["can_fuse_qnorm", "visionhope_qnorm"])):
        for n in names:
            assert hasattr(mod, n), (mod.__name__, n)


def test_reference_srnl_over_dropin_rejects_cpu_inputs():
    ref = reference("dropin")
    m = ref.SRNL(32, 16, directions=1)
    with pytest.raises(ValueError, match="same CUDA device"):
        m(torch.randn(1, 10, 32))


@pytest.mark.parametrize("name", ["visionhope_tiny", "visionhope_base"])
def test_harness_loads_reference_state_dict(name):
    from visionhope_b200.backbone import create_model

    ref = reference("native")
    torch.manual_seed(3)
    sd = ref.create_model(name).state_dict()
    ours = create_model(name)
    missing, unexpected = ours.load_state_dict(sd, strict=True)
    assert not missing and not unexpected
    theirs = {k: tuple(v.shape) for k, v in sd.items()}
    assert {k: tuple(v.shape) for k, v in ours.state_dict().items()} == theirs


@pytest.mark.parametrize("arch,out_norm", [("tiny", True), ("base", False)])
def test_dense_backbone_loads_reference_adapter_state_dict(arch, out_norm):
    """DenseBackbone keeps the parameter names of tasks/backbone.py's VisionHOPEBackbone
    (downsample_layers, stages, out_norms) and its argument checks."""
    import importlib

    from visionhope_b200.backbone import DenseBackbone

    reference("native")
    tb = importlib.import_module("visionhope.tasks.backbone")
    torch.manual_seed(3)
    sd = tb.VisionHOPEBackbone(arch, out_norm=out_norm).state_dict()
    ours = DenseBackbone(arch, out_norm=out_norm)
    missing, unexpected = ours.load_state_dict(sd, strict=True)
    assert not missing and not unexpected
    for bad in ({"arch": "huge"}, {"out_indices": (1, 0)}, {"out_indices": (0, 4)}, {"out_indices": ()}):
        args = {"arch": "tiny", **bad}
        with pytest.raises(ValueError):
            DenseBackbone(**args)
        with pytest.raises(ValueError):
            tb.VisionHOPEBackbone(**args)
