"""The four-direction VisionHOPE operator on B200 (mirror of models/operator.py).

Same constructor, parameters, path selection and results as the reference.  The fast
spatial path differs in how it feeds the kernel, not in what it computes: instead of
materialising four serialized copies of x and of the queries (operator.py:79-86, 66-70)
it hands the fused kernel the channels-last image and the single W_q projection, and the
kernel applies each scan's index map while loading.
"""
import torch
from torch import nn

from .srnl import SRNL, trunc_normal_
from .utils.cuda import on_tensor_device
from .utils.direction_fusion import visionhope_postprocess_scale
from .utils.inference import linear_cached


class VisionHOPEOperator(nn.Module):
    """Serialize four scans, apply SRNL, and restore/fuse the spatial outputs."""

    def __init__(self, dim, head_dim=16, chunk_size=None, direction_merge="scale",
                 share_direction_skip=True, *, fast_inference=False, _initialize=True):
        super().__init__()
        if not isinstance(share_direction_skip, bool):
            raise TypeError("share_direction_skip must be a bool")
        if direction_merge not in {"sum", "scale", "softmax"}:
            raise ValueError("direction_merge must be sum, scale, or softmax")
        self.dim = int(dim)
        self.head_dim = int(head_dim)
        self.share_direction_skip = share_direction_skip
        self.direction_merge = direction_merge
        self.srnl = SRNL(dim, head_dim, chunk_size, directions=4,
                         fast_inference=fast_inference, _initialize=False)
        self.num_heads = self.srnl.num_heads
        self.W_q = nn.Linear(dim, dim)
        skip_shape = (self.num_heads, head_dim) if share_direction_skip else (4, self.num_heads, head_dim)
        self.d_skip = nn.Parameter(torch.zeros(skip_shape))
        self.direction_scale = nn.Parameter(torch.ones(4, dim)) if direction_merge == "scale" else None
        self.direction_logits = nn.Parameter(torch.zeros(4, dim)) if direction_merge == "softmax" else None
        if _initialize:
            self.reset_parameters()

    @property
    def fast_inference(self):
        return self.srnl.fast_inference

    @fast_inference.setter
    def fast_inference(self, enabled):
        self.srnl.fast_inference = enabled

    def reset_parameters(self):
        self.srnl.reset_parameters()
        trunc_normal_(self.W_q.weight, std=0.02)
        nn.init.zeros_(self.W_q.bias)
        nn.init.zeros_(self.d_skip)
        if self.direction_scale is not None:
            nn.init.ones_(self.direction_scale)
        if self.direction_logits is not None:
            nn.init.zeros_(self.direction_logits)

    def project_queries(self, seq_hw, height, width):
        q_hw = self.W_q(seq_hw)
        q_wh = q_hw.reshape(q_hw.shape[0], height, width, self.dim)
        q_wh = q_wh.transpose(1, 2).reshape_as(q_hw)
        return torch.stack((q_hw, q_hw.flip(1), q_wh, q_wh.flip(1)), dim=1)

    def direction_weights(self):
        if self.direction_merge == "scale":
            return self.direction_scale
        if self.direction_merge == "softmax":
            return 4.0 * torch.softmax(self.direction_logits, dim=0)
        return self.d_skip.new_ones((4, self.dim))

    @staticmethod
    def serialize(x, seq_hw=None):
        if seq_hw is None:
            seq_hw = x.flatten(2).transpose(1, 2)
        seq_wh = x.transpose(2, 3).flatten(2).transpose(1, 2)
        return torch.stack([
            seq_hw, torch.flip(seq_hw, dims=[1]), seq_wh, torch.flip(seq_wh, dims=[1])
        ], dim=1)

    def forward(self, x, *, channels_last=None):
        if x.ndim != 4 or x.shape[1] != self.dim:
            raise ValueError(f"VisionHOPEOperator expects [B, {self.dim}, H, W]")
        if channels_last is None:
            channels_last = x.is_contiguous(memory_format=torch.channels_last)
        path, _ = self._inference_path(x)
        if path != "ordinary":
            out = self._forward_fast(x, path).permute(0, 3, 1, 2)
            memory_format = torch.channels_last if channels_last else torch.contiguous_format
            return out.contiguous(memory_format=memory_format)
        return self._sequence_forward(x, channels_last)

    def _sequence_forward(self, x, channels_last, *, memories=None):
        batch_size, _, height, width = x.shape
        seq_hw = x.flatten(2).transpose(1, 2)
        xs = self.serialize(x, seq_hw)
        xc_multi = xs.view(batch_size, 4, xs.shape[2], self.num_heads, self.head_dim)
        xc_multi = xc_multi.transpose(2, 3).contiguous()
        q_raw = self.project_queries(seq_hw, height, width)
        if memories is None:
            y = self.srnl(xc_multi, q_raw, spatial_shape=(height, width))
        else:
            from .srnl_core.fused import srnl_sequence_inference

            y = srnl_sequence_inference(memories, xc_multi, q_raw, [self.srnl.chunk_size] * 4)
        weights = self.direction_weights()
        if y.dtype != xc_multi.dtype:
            y = y.to(xc_multi.dtype)
        return visionhope_postprocess_scale(y, xc_multi, self.d_skip.float(), weights.float(),
                                            height, width, channels_last)

    def _inference_path(self, x):
        if self.training:
            return "ordinary", "The operator is in training mode"
        query_dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype
        path, reason = self.srnl._inference_path(x, query_dtype)
        if path == "ordinary":
            return path, reason
        height, width = x.shape[-2:]
        chunk_size = self.srnl.chunk_size
        if chunk_size is None or chunk_size == height == width:
            return "spatial", None
        return "sequence", None

    def inference_status(self, x):
        """Report path selection for a valid NCHW input in the current context."""
        path, reason = self._inference_path(x)
        return {"path": path, "reason": reason}

    def _fusion_weights(self):
        if self.direction_merge == "softmax":
            return 4.0 * torch.softmax(self.direction_logits.detach().float(), dim=0)
        return self.direction_weights().detach().float()

    @on_tensor_device
    def _forward_fast(self, x, path, *, addend=None, final_dtype=None):
        """Inference-only fusion, returning contiguous NHWC fp32 for the output projection.

        On the spatial path, ``final_dtype`` makes the scan launch itself write
        ``(final_dtype)(out + addend)`` (``addend``: NHWC in x's dtype, e.g. the block's output
        position term) instead of the fp32 sum."""
        if torch.jit.is_tracing():
            raise RuntimeError("SRNL TorchScript tracing is unsupported; use eager or CUDA Graph inference.")
        if x.ndim != 4 or not x.is_cuda or x.shape[1] != self.dim or min(x.shape) <= 0:
            raise ValueError(f"Fused VisionHOPE expects nonempty CUDA [B, {self.dim}, H, W]")
        height, width = x.shape[-2:]
        memories = self.srnl._validate_memories(x.device)
        skip_shape = (self.num_heads, self.head_dim) if self.share_direction_skip else (4, self.num_heads, self.head_dim)
        if self.d_skip.shape != skip_shape or self.d_skip.device != x.device:
            raise ValueError("Directional skip has an invalid shape or device")
        for scale in (self.direction_scale, self.direction_logits):
            if scale is not None and (scale.shape != (4, self.dim) or scale.device != x.device):
                raise ValueError("Directional fusion weights have an invalid shape or device")
        if path == "sequence":
            out = self._sequence_forward(x, True, memories=memories).permute(0, 2, 3, 1).contiguous()
            if addend is not None:
                out = out + addend
            return out if final_dtype is None else out.to(final_dtype)
        from .srnl_core.fused import spatial_forward

        x_img = x.permute(0, 2, 3, 1)  # [B, H, W, C]; a view when x is channels-last
        if not x_img.is_contiguous():
            x_img = x_img.contiguous()
        q_img = linear_cached(self.W_q, x_img)
        if q_img.dtype != x_img.dtype:
            q_img = q_img.to(x_img.dtype)
        return spatial_forward(memories, x_img, q_img, self.d_skip, self._fusion_weights(),
                               int(height), int(width), self.head_dim, layout="image",
                               addend=addend, final_dtype=final_dtype)
