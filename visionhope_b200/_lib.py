"""ctypes binding of libvhope.so (the sm_100a kernels behind every public op).

There is no CPU or PyTorch fallback anywhere: if the library is missing, cannot be
loaded, or a tensor is not on a CUDA device, the call raises.  Status codes and the
thread-local message of ``vh_last_error`` surface as ``RuntimeError`` (the reference's
``TORCH_CHECK`` convention, models/srnl_core/csrc/fused.cu:136-168).
"""
from __future__ import annotations

import ctypes
import functools
import itertools
import os
import threading
from ctypes import c_float, c_int32, c_int64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libvhope.so"

VH_F32, VH_BF16, VH_F16 = 0, 1, 2
DTYPES = {torch.float32: VH_F32, torch.bfloat16: VH_BF16, torch.float16: VH_F16}
SUPPORTED_HEAD_DIMS = (4, 8, 16, 32, 64)


class VhConsts(ctypes.Structure):
    _fields_ = [("step_scale", c_float), ("min_retention", c_float), ("retention_bias", c_float),
                ("injection_margin", c_float), ("spectral_factor", c_float),
                ("spectral_clamp", c_int32)]


class VhMemories(ctypes.Structure):
    _fields_ = [("m", c_void_p), ("v", c_void_p), ("k", c_void_p), ("eta", c_void_p),
                ("alpha", c_void_p), ("per_chain", c_int32)]


class VhSpatialArgs(ctypes.Structure):
    _fields_ = [("mem", VhMemories), ("x", c_void_p), ("q", c_void_p),
                ("x_batch_stride", c_int64), ("x_dir_stride", c_int64), ("x_token_stride", c_int64),
                ("x_head_stride", c_int64),
                ("q_batch_stride", c_int64), ("q_dir_stride", c_int64), ("q_token_stride", c_int64),
                ("q_head_stride", c_int64),
                ("io_dtype", c_int32), ("remap", c_int32), ("skip", c_void_p),
                ("skip_per_dir", c_int32), ("weight", c_void_p), ("out", c_void_p),
                ("out_batch_stride", c_int64), ("batch", c_int32), ("height", c_int32),
                ("width", c_int32), ("heads", c_int32), ("head_dim", c_int32),
                ("consts", VhConsts), ("aux", c_void_p), ("addend", c_void_p),
                ("addend_batch_stride", c_int64), ("final_out", c_void_p),
                ("final_dtype", c_int32), ("final_batch_stride", c_int64)]


class VhSequenceArgs(ctypes.Structure):
    _fields_ = [("mem", VhMemories), ("x", c_void_p), ("q", c_void_p), ("y", c_void_p),
                ("x_dtype", c_int32), ("q_dtype", c_int32), ("q_mode", c_int32),
                ("batch", c_int32), ("dirs", c_int32), ("heads", c_int32), ("length", c_int32),
                ("head_dim", c_int32), ("chunk", c_int32 * 4), ("consts", VhConsts)]


class VhSequenceBwdArgs(ctypes.Structure):
    _fields_ = [("mem", VhMemories), ("x", c_void_p), ("q", c_void_p),
                ("x_dtype", c_int32), ("q_dtype", c_int32), ("q_mode", c_int32),
                ("grad_y", c_void_p), ("grad_x", c_void_p), ("grad_q", c_void_p), ("grad_m", c_void_p),
                ("grad_v", c_void_p), ("grad_k", c_void_p), ("grad_eta", c_void_p), ("grad_alpha", c_void_p),
                ("batch", c_int32), ("dirs", c_int32), ("heads", c_int32), ("length", c_int32),
                ("head_dim", c_int32), ("chunk", c_int32 * 4), ("consts", VhConsts)]


class VhDwconvArgs(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("gate", c_void_p), ("weight", c_void_p), ("bias", c_void_p),
                ("y", c_void_p), ("dtype", c_int32), ("mode", c_int32), ("ksize", c_int32),
                ("batch", c_int32), ("height", c_int32), ("width", c_int32), ("channels", c_int32),
                ("gate_dtype", c_int32), ("sumsq", c_void_p), ("pos_weight", c_void_p), ("pos_bias", c_void_p),
                ("pos_y", c_void_p), ("pos_ksize", c_int32)]


_lib = None
_lock = threading.Lock()
_inited = set()


def load() -> ctypes.CDLL:
    """Load libvhope.so once; raises if it has not been built (``python -m visionhope_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.is_file():
                raise RuntimeError(
                    f"libvhope.so is not built ({LIB_PATH}); run `python visionhope_b200/build.py`")
            lib = ctypes.CDLL(str(LIB_PATH))
            lib.vh_last_error.restype = ctypes.c_char_p
            lib.vh_version.restype = ctypes.c_char_p
            lib.vh_grn_workspace_bytes.restype = c_int64
            lib.vh_grn_workspace_bytes.argtypes = [c_int32] * 4
            for name in ("vh_srnl_spatial_fwd", "vh_srnl_sequence_fwd", "vh_qnorm_fwd",
                         "vh_dirfuse_fwd", "vh_grn_fwd", "vh_layernorm_fwd", "vh_init"):
                getattr(lib, name).restype = c_int32
            lib.vh_srnl_spatial_fwd.argtypes = [ctypes.POINTER(VhSpatialArgs), c_void_p]
            lib.vh_srnl_sequence_fwd.argtypes = [ctypes.POINTER(VhSequenceArgs), c_void_p]
            lib.vh_qnorm_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32,
                                         c_int32, c_int32, c_int32, c_void_p]
            lib.vh_dirfuse_fwd.argtypes = [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p,
                                           c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32,
                                           c_int32, c_void_p]
            lib.vh_grn_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_float, c_void_p,
                                       c_int32, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
                                       c_int32, c_int32, c_int32, c_void_p]
            lib.vh_layernorm_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_float,
                                             c_void_p, c_int32, c_void_p, c_void_p, c_int64, c_int32,
                                             c_void_p]
            lib.vh_init.argtypes = [c_int32]
            lib.vh_dwconv_fwd.restype = c_int32
            lib.vh_dwconv_fwd.argtypes = [ctypes.POINTER(VhDwconvArgs), c_void_p]
            lib.vh_dwconv_tiles.restype = c_int32
            lib.vh_dwconv_tiles.argtypes = [c_int32, c_int32]
            lib.vh_grn_apply_fwd.restype = c_int32
            lib.vh_grn_apply_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_float,
                                             c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32,
                                             c_void_p]
            lib.vh_rows_gemm_fwd.restype = c_int32
            lib.vh_rows_gemm_fwd.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
                                             c_void_p]
            lib.vh_ln_rows_gemm_fwd.restype = c_int32
            lib.vh_ln_rows_gemm_fwd.argtypes = [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                                c_int64, c_int32, c_int32, c_void_p]
            lib.vh_stem_conv_fwd.restype = c_int32
            lib.vh_stem_conv_fwd.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                             c_int32, c_int32, c_int32, c_void_p]
            lib.vh_add_cast_fwd.restype = c_int32
            lib.vh_add_cast_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p]
            lib.vh_bias_act_fwd.restype = c_int32
            lib.vh_bias_act_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int64, c_int32,
                                            c_int32, c_void_p]
            lib.vh_add_layernorm_fwd.restype = c_int32
            lib.vh_add_layernorm_fwd.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p,
                                                 c_void_p, c_float, c_void_p, c_int32, c_int64, c_int32,
                                                 c_void_p]
            lib.vh_last_launch_count.restype = c_int32
            lib.vh_last_launch_count.argtypes = []
            lib.vh_tc_status.restype = c_int32
            lib.vh_tc_status.argtypes = [c_int32]
            lib.vh_probe_ffma.restype = c_int32
            lib.vh_probe_ffma.argtypes = [c_void_p, c_int32, c_int32, c_void_p]
            # backward (training) entry points
            lib.vh_qnorm_bwd.restype = c_int32
            lib.vh_qnorm_bwd.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32] + [c_int32] * 5 + [c_void_p]
            lib.vh_dirfuse_bwd_workspace_bytes.restype = c_int64
            lib.vh_dirfuse_bwd_workspace_bytes.argtypes = [c_int32] * 5
            lib.vh_dirfuse_bwd.restype = c_int32
            lib.vh_dirfuse_bwd.argtypes = ([c_void_p] + [c_int64] * 4 + [c_void_p, c_void_p, c_int32, c_void_p, c_int32,
                                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64]
                                           + [c_int32] * 5 + [c_void_p])
            lib.vh_layernorm_bwd_workspace_bytes.restype = c_int64
            lib.vh_layernorm_bwd_workspace_bytes.argtypes = [c_int64, c_int32]
            lib.vh_layernorm_bwd.restype = c_int32
            lib.vh_layernorm_bwd.argtypes = ([c_void_p, c_void_p, c_int32] + [c_void_p] * 7 + [c_int64, c_int64, c_int32,
                                             c_void_p])
            lib.vh_srnl_sequence_bwd_workspace_bytes.restype = c_int64
            lib.vh_srnl_sequence_bwd_workspace_bytes.argtypes = [ctypes.POINTER(VhSequenceBwdArgs)]
            lib.vh_srnl_sequence_bwd.restype = c_int32
            lib.vh_srnl_sequence_bwd.argtypes = [ctypes.POINTER(VhSequenceBwdArgs), c_void_p, c_int64, c_void_p]
            lib.vh_grn_bwd_workspace_bytes.restype = c_int64
            lib.vh_grn_bwd_workspace_bytes.argtypes = [c_int32, c_int32]
            lib.vh_grn_bwd.restype = c_int32
            lib.vh_grn_bwd.argtypes = ([c_void_p, c_void_p, c_int32] + [c_void_p] * 7 + [c_int64] + [c_int32] * 4
                                       + [c_void_p])
            lib.vh_residual_add_fwd.restype = c_int32
            lib.vh_residual_add_fwd.argtypes = ([c_void_p, c_int32, c_void_p, c_int32] + [c_void_p] * 3
                                                + [c_int32, c_int64, c_int32, c_void_p])
            lib.vh_residual_add_bwd_workspace_bytes.restype = c_int64
            lib.vh_residual_add_bwd_workspace_bytes.argtypes = [c_int64, c_int32]
            lib.vh_residual_add_bwd.restype = c_int32
            lib.vh_residual_add_bwd.argtypes = ([c_void_p, c_void_p, c_int32] + [c_void_p] * 5
                                                + [c_int64, c_int32, c_int64, c_int32, c_void_p])
            _lib = lib
    return _lib


def version() -> str:
    return load().vh_version().decode()


# Kernels the library launched through this module (the library reports each call's count).
launch_count = 0


def check(rc: int, what: str) -> None:
    """Raise on a non-zero status; otherwise count the kernels the call launched."""
    global launch_count
    lib = load()
    if rc != 0:
        msg = lib.vh_last_error().decode() or "unknown error"
        raise RuntimeError(f"{what} failed ({rc}): {msg}")
    launch_count += lib.vh_last_launch_count()


def ensure_device(t: torch.Tensor) -> None:
    """Require a CUDA tensor and make sure its device has been initialised for the library."""
    if not t.is_cuda:
        raise RuntimeError("VisionHOPE B200 kernels require CUDA tensors (no CPU path exists)")
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if dev not in _inited:
        with torch.cuda.device(dev):
            check(load().vh_init(dev), "vh_init")
        _inited.add(dev)


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPES[dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {dtype}; use float32, bfloat16 or float16") from exc


def consts(step_scale, min_retention, retention_bias, injection_margin, spectral_margin,
           spectral_clamp=True) -> VhConsts:
    return VhConsts(float(step_scale), float(min_retention), float(retention_bias),
                    float(injection_margin), float(2.0 * spectral_margin), int(bool(spectral_clamp)))


def memories(states, per_chain: bool = False) -> VhMemories:
    m, v, k, e, a = states
    return VhMemories(m.data_ptr(), v.data_ptr(), k.data_ptr(), e.data_ptr(), a.data_ptr(),
                      int(per_chain))


def env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) not in ("", "0", "false", "False")


def on_input_device(fn):
    """Decorator: run ``fn`` with the device of its first CUDA tensor argument current, so that
    ``stream_handle()`` and torch allocations inside refer to the inputs' GPU.  Calls whose
    inputs are all on the current device (or on no GPU, which the entry points then reject)
    run unchanged."""
    @functools.wraps(fn)
    def call(*args, **kwargs):
        for value in itertools.chain(args, kwargs.values()):
            if isinstance(value, torch.Tensor) and value.is_cuda:
                if value.device.index != torch.cuda.current_device():
                    with torch.cuda.device(value.device):
                        return fn(*args, **kwargs)
                break
        return fn(*args, **kwargs)
    return call
