"""VisionHOPE backbone assembly used to drive the hot path end to end (configs 4 and 5).

This is caller code, not part of the hot path: it wires cuDNN convolutions, cuBLAS
projections and BatchNorm around the library's operator, LayerNorm and GRN so that
whole-model throughput can be measured.  Parameter names and shapes match the
reference's modules (models/block.py, models/layers.py, models/hierarchical.py,
models/factory.py) so a reference state_dict loads unchanged; the forward order of
every block follows models/block.py:63-106 and the prepared fast branch block.py:73-80.
Every LayerNorm, GRN and SRNL operator call runs on libvhope.so.
"""
from __future__ import annotations

from copy import deepcopy

import torch
from torch import nn
from torch.nn import functional as F

from .mixer import ScanMemories, ScanMixer
from .utils.grn import GlobalResponseNorm
from .utils.bias_act import add_cast, add_cast_ok, bias_act, stem_conv, stem_conv_ok
from .utils.dwconv import depthwise_fused, fusable, gate_pos_ok
from .utils.grn_cuda import grn_apply, grn_apply_ok, grn_forward
from .utils.inference import cache_half_weights, linear_cached, norm_linear_cached
from .utils.layer_norm_cuda import add_layernorm_rows, layernorm_rows


# (in, out) channels of proj_in where norm1 runs as the projection's prologue: the stage-1 and
# stage-2 shapes of VisionHOPE-T, narrow enough for the row GEMM.
_NORM1_PROJ_IN_FUSED = {(64, 32), (128, 64)}


def _autocast_dtype():
    """The CUDA autocast dtype when autocast is on, else None."""
    return torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else None

MODEL_CONFIGS = {
    "visionhope_tiny": dict(embed_dims=(64, 128, 256, 512), mixer_dims=(32, 64, 128, 256),
                            depths=(3, 4, 18, 4)),
    "visionhope_small": dict(embed_dims=(64, 160, 320, 512), mixer_dims=(32, 80, 160, 256),
                             depths=(4, 8, 25, 8)),
    "visionhope_base": dict(embed_dims=(96, 192, 448, 640), mixer_dims=(48, 96, 224, 320),
                            depths=(4, 8, 25, 8)),
}


def pointwise(conv, x):
    """A 1x1 convolution of a channels-last NCHW tensor as a GEMM over its NHWC view.

    The GEMM applies the bias in its epilogue; a convolution of a channels-last tensor adds
    the bias in a separate broadcast pass.  Other layouts use the convolution itself."""
    if x.is_cuda and x.is_contiguous(memory_format=torch.channels_last) and x.shape[1] > 1:
        return linear_cached(conv, x.permute(0, 2, 3, 1)).permute(0, 3, 1, 2)
    return conv(x)


def _is_exact_gelu(m):
    return isinstance(m, nn.GELU) and m.approximate == "none"


class LayerNorm2d(nn.Module):
    """LayerNorm over the channels of an NCHW tensor; fp32 output in channels-last storage.

    Replaces models/layers.py:9-35: both the Triton path and the ``inference_layout``
    F.layer_norm path map to ``vh_layernorm_fwd``.
    """

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim))
        self.eps = eps
        self.inference_layout = False
        # Set when the only consumer is a convolution that autocast runs in lower precision:
        # the kernel then writes that dtype directly (the fp32 result rounded once, exactly
        # the cast autocast would apply), saving a separate cast pass.
        self.emit_autocast_dtype = False

    def forward(self, x):
        b, c, h, w = x.shape
        rows = x.permute(0, 2, 3, 1)
        if not rows.is_contiguous():
            rows = rows.contiguous()
        out_dtype = torch.float32
        if self.emit_autocast_dtype and _autocast_dtype() in (torch.bfloat16, torch.float16):
            out_dtype = _autocast_dtype()
        y = layernorm_rows(rows.reshape(b * h * w, c), self.weight, self.bias, self.eps, out_dtype=out_dtype)
        return y.view(b, h, w, c).permute(0, 3, 1, 2)

    def forward_add(self, x, r, inplace=False):
        """(x + r, LayerNorm(x + r)) for a channels-last CUDA x and r of its shape: the residual
        add and this norm in one pass (the sum goes into x itself when ``inplace``).  Falls
        back to the two operations when the fused kernel does not apply."""
        b, c, h, w = x.shape
        if (x.is_cuda and not torch.is_grad_enabled() and c % 8 == 0 and c <= 2048
                and x.dtype in (torch.float32, torch.bfloat16) and r.dtype in (torch.float32, torch.bfloat16)
                and torch.promote_types(x.dtype, r.dtype) == x.dtype and r.shape == x.shape
                and x.is_contiguous(memory_format=torch.channels_last)
                and r.is_contiguous(memory_format=torch.channels_last)):
            out_dtype = torch.float32
            if self.emit_autocast_dtype and _autocast_dtype() in (torch.bfloat16, torch.float16):
                out_dtype = _autocast_dtype()
            s = x if inplace else torch.empty_like(x, memory_format=torch.channels_last)
            rows = lambda t: t.permute(0, 2, 3, 1).reshape(b * h * w, c)
            _, y = add_layernorm_rows(rows(x), rows(r), self.weight, self.bias, self.eps, out_dtype=out_dtype,
                                      sum_out=rows(s))
            return s, y.view(b, h, w, c).permute(0, 3, 1, 2)
        x = x + r
        return x, self(x)


def build_norm(dim, norm_layer="group"):
    if norm_layer == "group":
        return nn.GroupNorm(1, dim)
    if norm_layer == "layernorm2d":
        return LayerNorm2d(dim)
    raise ValueError(f"Unsupported norm_layer={norm_layer!r}.")


class FeedForwardNetwork(nn.Module):
    """1x1 expand, GELU, residual depthwise 3x3 + GELU, GRN (fp32), 1x1 project."""

    def __init__(self, in_features, hidden_features=None, out_features=None, act_layer=nn.GELU,
                 drop=0.0, use_grn=False, use_dwconv=False):
        super().__init__()
        hidden_features = hidden_features or in_features
        out_features = out_features or in_features
        self.fc1 = nn.Conv2d(in_features, hidden_features, kernel_size=1)
        self.act = act_layer()
        self.use_dwconv = use_dwconv
        self.dwconv = (nn.Conv2d(hidden_features, hidden_features, kernel_size=3, padding=1,
                                 groups=hidden_features) if use_dwconv else nn.Identity())
        self.dwconv_act = act_layer() if use_dwconv else nn.Identity()
        self.grn = GlobalResponseNorm(hidden_features) if use_grn else nn.Identity()
        self.fc2 = nn.Conv2d(hidden_features, out_features, kernel_size=1)
        self.drop = nn.Dropout(drop)

    def forward(self, x):
        x = pointwise(self.fc1, x)
        sumsq = None
        if (self.use_dwconv and _is_exact_gelu(self.act) and _is_exact_gelu(self.dwconv_act)
                and fusable(x, self.dwconv)):
            # gelu(fc1), the depthwise convolution, its residual and the second gelu in one pass;
            # with GRN next, the same pass also sums y^2 per channel over each pixel tile
            stats = isinstance(self.grn, GlobalResponseNorm) and grn_apply_ok(x)
            x = depthwise_fused(x, self.dwconv, "gelu", with_sumsq=stats)
            if stats:
                x, sumsq = x
        else:
            x = self.act(x)
            if self.use_dwconv:
                x = self.dwconv_act(x + self.dwconv(x))
        ac = _autocast_dtype()
        if isinstance(self.grn, GlobalResponseNorm) and ac in (torch.bfloat16, torch.float16) and x.is_cuda:
            # fc2 runs under autocast and casts GRN's fp32 output to `ac`; emit it directly.
            if not x.is_contiguous(memory_format=torch.channels_last):
                x = x.contiguous(memory_format=torch.channels_last)
            if sumsq is not None:
                x = grn_apply(x, sumsq, self.grn.gamma, self.grn.beta, self.grn.eps, out_dtype=ac)
            else:
                x = grn_forward(x, self.grn.gamma, self.grn.beta, self.grn.eps, out_dtype=ac)
        else:
            x = self.grn(x)
        return self.drop(pointwise(self.fc2, self.drop(x)))


def _fused_epilogue_ok(x):
    """bf16 autocast inference on a channels-last CUDA input: the folded stem and downsample
    layers then run their bias/GELU epilogue as one kernel."""
    return (x.is_cuda and not torch.is_grad_enabled() and _autocast_dtype() == torch.bfloat16
            and x.is_contiguous(memory_format=torch.channels_last))


def _fold_conv_bn(conv, bn):
    """conv followed by eval-mode bn -> conv with w * g / sqrt(var + eps), (b - mean) * that + beta."""
    scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
    conv.weight.mul_(scale.view(-1, 1, 1, 1).to(conv.weight.dtype))
    bias = conv.bias if conv.bias is not None else torch.zeros_like(bn.running_mean)
    folded = (bias - bn.running_mean) * scale + bn.bias
    if conv.bias is None:
        conv.bias = nn.Parameter(folded.to(conv.weight.dtype))
    else:
        conv.bias.copy_(folded)


class PatchEmbedding(nn.Module):
    """Stride-4 convolutional stem: conv/BN/GELU x3 then conv/BN (layers.py:85-107)."""

    def __init__(self, in_chans, embed_dim, patch_size=4):
        super().__init__()
        if patch_size != 4:
            raise ValueError("The VisionHOPE stem requires patch_size=4")
        widths = [embed_dim // 2, embed_dim // 2, embed_dim, embed_dim]
        strides = [2, 1, 2, 1]
        if min(widths) <= 0:
            raise ValueError("embed_dim is too small for the convolutional stem")
        layers = []
        for i, (width, stride) in enumerate(zip(widths, strides)):
            layers += [nn.Conv2d(in_chans, width, 3, stride=stride, padding=1), nn.BatchNorm2d(width)]
            if i < 3:
                layers.append(nn.GELU())
            in_chans = width
        self.proj = nn.Sequential(*layers)
        self.norm = nn.Identity()

    def forward(self, x):
        plan = getattr(self, "_folded_plan", None)
        if plan is not None and _fused_epilogue_ok(x):
            # Folded convolutions with the bias (and GELU) applied by one pointwise kernel in
            # fp32: GELU outputs in the autocast dtype (the next convolution's input), the
            # last layer in fp32, the dtype BatchNorm produced (the residual stream's).
            for i, (conv, gelu) in enumerate(plan):
                out_dtype = _autocast_dtype() if gelu else torch.float32
                if i == 0 and out_dtype in (torch.bfloat16, torch.float32) and stem_conv_ok(x, conv):
                    # the 3-channel first layer: convolution, bias and GELU in one kernel
                    x = stem_conv(x, conv, "gelu" if gelu else None, out_dtype=out_dtype)
                    continue
                y = F.conv2d(x, conv.weight, None, conv.stride, conv.padding)
                x = bias_act(y, conv.bias, "gelu" if gelu else None, out_dtype=out_dtype)
            return self.norm(x)
        return self.norm(self.proj(x))

    @torch.no_grad()
    def fold_batchnorm(self):
        """Inference: fold each eval-mode BatchNorm into the convolution before it."""
        layers, n = list(self.proj), 0
        for i in range(len(layers) - 1):
            if isinstance(layers[i], nn.Conv2d) and isinstance(layers[i + 1], nn.BatchNorm2d):
                _fold_conv_bn(layers[i], layers[i + 1])
                layers[i + 1] = nn.Identity()
                n += 1
        self.proj = nn.Sequential(*layers)
        plan = []
        for i, layer in enumerate(layers):
            if isinstance(layer, nn.Conv2d):
                nxt = [m for m in layers[i + 1:i + 3] if not isinstance(m, nn.Identity)]
                plan.append((layer, bool(nxt) and _is_exact_gelu(nxt[0])))
        if all(conv.bias is not None and conv.out_channels % 8 == 0 for conv, _ in plan):
            self._folded_plan = plan
        return n


class Downsample(nn.Module):
    def __init__(self, in_dim, out_dim):
        super().__init__()
        self.proj = nn.Conv2d(in_dim, out_dim, 3, stride=2, padding=1, bias=False)
        self.norm = nn.BatchNorm2d(out_dim)

    def forward(self, x, pending=None):
        """Downsample x (+ pending: the previous stage's last residual branch, added first)."""
        if getattr(self, "_folded", False) and self.proj.out_channels % 8 == 0 and _fused_epilogue_ok(x):
            if pending is not None:
                # the stage's last residual add and autocast's bf16 cast of the sum in one pass
                x = add_cast(x, pending, torch.bfloat16) if add_cast_ok(x, pending) else x + pending
            y = F.conv2d(x, self.proj.weight, None, self.proj.stride, self.proj.padding)
            return bias_act(y, self.proj.bias, None, out_dtype=torch.float32)  # BatchNorm's dtype
        if pending is not None:
            x = x + pending
        return self.norm(self.proj(x))

    @torch.no_grad()
    def fold_batchnorm(self):
        """Inference: fold the eval-mode BatchNorm into the convolution."""
        if not isinstance(self.norm, nn.BatchNorm2d):
            return 0
        _fold_conv_bn(self.proj, self.norm)
        self.norm = nn.Identity()
        self._folded = True
        return 1


class VisionHOPEBlock(nn.Module):
    """cpe -> norm1 -> local features -> operator (+ output position conv) -> proj_out -> residual,
    then norm2 -> FFN(GRN) -> residual, with optional LayerScale (models/block.py:13-106)."""

    def __init__(self, dim, head_dim=16, chunk_size=None, mlp_ratio=4.0, drop_path=0.0,
                 mixer_dim=None, local_mode="gated_dwconv7", norm_layer="layernorm2d",
                 layer_scale_init_value=1e-6, use_grn=True, use_mlp_dwconv=True,
                 use_direction_scale=True, direction_merge="sum", use_block_cpe=True,
                 use_output_lepe=True, share_direction_skip=True):
        super().__init__()
        mixer_dim = int(mixer_dim) if mixer_dim is not None else dim
        if local_mode not in {"gated_dwconv7", "residual_dwconv", "silu_dwconv"}:
            raise ValueError("Unsupported local_mode")
        self.dim, self.mixer_dim, self.local_mode = dim, mixer_dim, local_mode
        self._inference_prepared = False
        self.cpe = nn.Conv2d(dim, dim, 3, padding=1, groups=dim) if use_block_cpe else None
        self.norm1 = build_norm(dim, norm_layer)
        self.proj_in = nn.Conv2d(dim, mixer_dim, 1)
        if use_direction_scale and direction_merge == "sum":
            direction_merge = "scale"
        if chunk_size is not None:
            raise NotImplementedError("the harness runs image-aligned chunks (chunk_size=None) only")
        self.operator = ScanMixer(mixer_dim, head_dim, direction_merge, share_direction_skip)
        k = 7 if local_mode == "gated_dwconv7" else 3
        self.local_conv = nn.Conv2d(mixer_dim, mixer_dim, k, padding=k // 2, groups=mixer_dim)
        self.local_gate = nn.Conv2d(mixer_dim, mixer_dim, 1) if local_mode == "gated_dwconv7" else None
        self.local_act = nn.SiLU() if local_mode == "silu_dwconv" else nn.Identity()
        self.local_position = (nn.Conv2d(mixer_dim, mixer_dim, 5, padding=2, groups=mixer_dim)
                               if use_output_lepe else None)
        self.proj_out = nn.Linear(mixer_dim, dim)
        nn.init.trunc_normal_(self.proj_out.weight, std=0.02, a=-2.0, b=2.0)
        nn.init.zeros_(self.proj_out.bias)
        self.drop_path = nn.Identity()  # inference only: stochastic depth is the identity
        self.drop_path_rate = float(drop_path)
        self.norm2 = build_norm(dim, norm_layer)
        self.ffn = FeedForwardNetwork(dim, int(dim * mlp_ratio), use_grn=use_grn, use_dwconv=use_mlp_dwconv)
        if layer_scale_init_value is not None and layer_scale_init_value > 0.0:
            self.gamma1 = nn.Parameter(layer_scale_init_value * torch.ones(dim, 1, 1))
            self.gamma2 = nn.Parameter(layer_scale_init_value * torch.ones(dim, 1, 1))
        else:
            self.gamma1 = None
            self.gamma2 = None

    def _norm1_proj_in(self, x):
        """proj_in(norm1(x)) as one kernel (the LayerNorm as the row GEMM's prologue) for the
        prepared block under bf16 autocast, at the projection shapes where that measured faster
        than the two passes; None elsewhere."""
        if not (self._inference_prepared and isinstance(self.norm1, LayerNorm2d) and x.is_cuda
                and x.is_contiguous(memory_format=torch.channels_last)
                and (self.proj_in.in_channels, self.proj_in.out_channels) in _NORM1_PROJ_IN_FUSED):
            return None
        inner = norm_linear_cached(self.norm1, self.proj_in, x.permute(0, 2, 3, 1))
        return None if inner is None else inner.permute(0, 3, 1, 2)

    def _local_features(self, x, inner=None):
        return self._local_and_position(x, inner, False)[0]

    def _local_and_position(self, x, inner, want_position):
        """(x_local, position term or None).  With ``want_position``, the gated local features
        and the output position term conv5x5(x_local) + b come from one depthwise kernel where
        it applies (whole 14 x 14 or 7 x 7 images, bf16); the term is NHWC in x_local's dtype."""
        if inner is None:
            inner = pointwise(self.proj_in, x)
        if self.local_mode == "gated_dwconv7":
            gate = pointwise(self.local_gate, inner)
            if fusable(inner, self.local_conv) and gate.dtype == inner.dtype:
                if (want_position and self.local_position is not None
                        and gate_pos_ok(inner, self.local_conv, self.local_position)):
                    x_local, pos = depthwise_fused(inner, self.local_conv, "gate_pos", gate=gate,
                                                   pos_conv=self.local_position)
                    return x_local, pos.permute(0, 2, 3, 1)
                return depthwise_fused(inner, self.local_conv, "gate", gate=gate), None
            return inner + torch.sigmoid(gate) * self.local_conv(inner), None
        conv = self.local_act(self.local_conv(inner))
        return (conv if self.local_mode == "silu_dwconv" else inner + conv), None

    def spatial_branch(self, x, *, inner=None):
        """The mixer branch on x = norm1(block input); ``inner`` = proj_in(x) when the caller
        already computed it (then x only supplies the memory format)."""
        channels_last = x.is_contiguous(memory_format=torch.channels_last)
        x_local, lepe = self._local_and_position(x, inner, self._inference_prepared)
        if self._inference_prepared and x_local.dtype == (_autocast_dtype() or x_local.dtype):
            # The reference's prepared fast branch (block.py:73-80): the scan launch adds the
            # output position term and writes the dtype the output projection consumes,
            # (out + lepe) rounded once, as the reference's fp32 add followed by autocast's cast.
            if lepe is None and self.local_position is not None:
                if fusable(x_local, self.local_position):
                    lepe = depthwise_fused(x_local, self.local_position, "bias").permute(0, 2, 3, 1)
                else:
                    lepe = self.local_position(x_local).permute(0, 2, 3, 1)
            out = self.operator(x_local, addend=lepe, out_dtype=_autocast_dtype() or torch.float32)
            out = linear_cached(self.proj_out, out)
            # NHWC storage viewed as NCHW (channels-last); the reference copies it to
            # contiguous NCHW here, which only costs a layout pass before the residual add.
            out = out.permute(0, 3, 1, 2)
            return out if channels_last else out.contiguous()
        # The unprepared order (block.py:82-88): fp32 operator output, the position term added
        # in NCHW, then proj_out as a 1x1 convolution.
        out = self.operator(x_local).permute(0, 3, 1, 2)
        if self.local_position is not None:
            out = out + self.local_position(x_local)
        out = F.conv2d(out, self.proj_out.weight[:, :, None, None], self.proj_out.bias)
        return out.contiguous(memory_format=torch.channels_last if channels_last else torch.contiguous_format)

    @staticmethod
    def _residual(x, branch, gamma):
        return x + branch if gamma is None else x + gamma * branch

    def forward(self, x):
        x, pending = self.forward_deferred(x)
        return x if pending is None else x + pending

    def forward_deferred(self, x, pending=None):
        """The block on x + pending, returning (x', r) whose sum is the block's output: the
        last residual add is left to the next block, whose cpe adds it while reading its
        input.  pending is None for the first block of a stage."""
        if self.training and self._inference_prepared:
            raise RuntimeError("A block with folded LayerScale weights cannot be trained")
        if self.cpe is not None:
            if fusable(x, self.cpe) and (pending is None or pending.is_contiguous(memory_format=torch.channels_last)):
                x = depthwise_fused(x, self.cpe, "resid", addend=pending)
            else:
                x = x if pending is None else x + pending
                x = x + self.cpe(x)
        elif pending is not None:
            x = x + pending
        inner = self._norm1_proj_in(x)
        branch = self.spatial_branch(self.norm1(x)) if inner is None else self.spatial_branch(x, inner=inner)
        if self.gamma1 is None and isinstance(self.norm2, LayerNorm2d):
            # x + branch and norm2 in one pass; x is this block's own tensor once cpe ran
            x, n2 = self.norm2.forward_add(x, branch, inplace=self.cpe is not None)
        else:
            x = self._residual(x, branch, self.gamma1)
            n2 = self.norm2(x)
        ffn = self.ffn(n2)
        if self.gamma2 is not None:
            return x + self.gamma2 * ffn, None
        return x, ffn


def initialize_weights(module):
    if isinstance(module, (nn.Linear, nn.Conv2d)):
        nn.init.trunc_normal_(module.weight, std=0.02, a=-2.0, b=2.0)
        if module.bias is not None:
            nn.init.constant_(module.bias, 0)


class HierarchicalVisionHOPE(nn.Module):
    """Four-stage VisionHOPE with the projection classifier head (models/hierarchical.py:11-85)."""

    def __init__(self, in_chans=3, num_classes=1000, embed_dims=(64, 128, 256, 512),
                 mixer_dims=(32, 64, 128, 256), depths=(3, 4, 18, 4), chunk_sizes=None,
                 mlp_ratios=(4.0, 4.0, 4.0, 4.0), head_dim=16, img_size=None, drop_path_rate=0.1,
                 local_mode="gated_dwconv7", norm_layer="layernorm2d", layer_scale_init_value=1e-6,
                 use_grn=True, use_mlp_dwconv=True, use_direction_scale=True, direction_merge="sum",
                 use_block_cpe=True, use_output_lepe=True, projection_dim=1024,
                 share_direction_skip=True):
        super().__init__()
        self.num_classes = num_classes
        self.embed_dims = list(embed_dims)
        self.mixer_dims = list(mixer_dims) if mixer_dims is not None else list(embed_dims)
        self.depths = list(depths)
        self.chunk_sizes = [None] * 4 if chunk_sizes is None else list(chunk_sizes)
        self.head_dim = int(head_dim)
        self.img_size = img_size
        if isinstance(mlp_ratios, (int, float)):
            mlp_ratios = [float(mlp_ratios)] * 4
        if any(len(v) != 4 for v in (self.embed_dims, self.mixer_dims, self.depths, self.chunk_sizes,
                                     mlp_ratios)):
            raise ValueError("Hierarchical VisionHOPE requires four stage configurations")
        self.downsample_layers = nn.ModuleList([PatchEmbedding(in_chans, embed_dims[0])])
        for i in range(3):
            self.downsample_layers.append(Downsample(embed_dims[i], embed_dims[i + 1]))
        rates = [v.item() for v in torch.linspace(0, drop_path_rate, sum(depths))]
        self.stages = nn.ModuleList()
        offset = 0
        for i in range(4):
            self.stages.append(nn.Sequential(*[
                VisionHOPEBlock(dim=embed_dims[i], head_dim=head_dim, chunk_size=self.chunk_sizes[i],
                                mlp_ratio=mlp_ratios[i], drop_path=rates[offset + j],
                                mixer_dim=self.mixer_dims[i], local_mode=local_mode,
                                norm_layer=norm_layer, layer_scale_init_value=layer_scale_init_value,
                                use_grn=use_grn, use_mlp_dwconv=use_mlp_dwconv,
                                use_direction_scale=use_direction_scale, direction_merge=direction_merge,
                                use_block_cpe=use_block_cpe, use_output_lepe=use_output_lepe,
                                share_direction_skip=share_direction_skip)
                for j in range(depths[i])]))
            offset += depths[i]
        self.norm = build_norm(embed_dims[-1], norm_layer)
        self.head_pre_logits = nn.Conv2d(embed_dims[-1], projection_dim, 1)
        self.head_norm = nn.BatchNorm2d(projection_dim)
        self.head_act = nn.SiLU()
        self.num_features = int(projection_dim)
        self.head = nn.Linear(self.num_features, num_classes)
        self.apply(initialize_weights)

    @staticmethod
    def _run_stage(stage, x):
        """The stage's blocks with each block's last residual add carried into the next block's
        cpe (one fused pass).  Returns (x, pending): the stage's output is x + pending (pending
        None when nothing is left to add), so its consumer can fuse the final add."""
        pending = None
        for blk in stage:
            if isinstance(blk, VisionHOPEBlock):
                x, pending = blk.forward_deferred(x, pending)
            else:
                x = blk(x if pending is None else x + pending)
                pending = None
        return x, pending

    def forward_intermediates(self, x):
        outs = []
        for down, stage in zip(self.downsample_layers, self.stages):
            x, pending = self._run_stage(stage, down(x))
            x = x if pending is None else x + pending
            outs.append(x)
        return tuple(outs)

    def forward_features(self, x):
        pending = None
        for i, (down, stage) in enumerate(zip(self.downsample_layers, self.stages)):
            if i == 0 or isinstance(down, Downsample):
                x = down(x) if pending is None else down(x, pending)
            else:
                x = down(x if pending is None else x + pending)
            x, pending = self._run_stage(stage, x)
        if pending is not None and isinstance(self.norm, LayerNorm2d):
            _, n = self.norm.forward_add(x, pending)  # the last residual add and the final norm
        else:
            n = self.norm(x if pending is None else x + pending)
        x = self.head_act(self.head_norm(self.head_pre_logits(n)))
        return x.mean(dim=[2, 3])

    def forward(self, x):
        return self.head(self.forward_features(x))


class DenseBackbone(nn.Module):
    """Stage features for detection and segmentation necks (tasks/backbone.py:19-125): the
    hierarchical backbone's downsample layers and stages, then one LayerNorm2d per stage
    (``out_norms``) on the features of ``out_indices``.  Parameter names match the reference's
    ``VisionHOPEBackbone``, so its state_dict loads with strict=True.  Each returned stage's last
    residual add runs fused with its output norm (``LayerNorm2d.forward_add``: one pass gives
    the stage output, which the next downsample reads, and its normalized copy).  Loading
    ImageNet weights, frozen stages and activation checkpointing stay with the caller (training
    options of the reference's adapter)."""

    def __init__(self, arch="tiny", in_chans=3, out_indices=(0, 1, 2, 3), out_norm=True, channels_last=True,
                 **kwargs):
        super().__init__()
        if arch not in {"tiny", "small", "base"}:
            raise ValueError("arch must be 'tiny', 'small', or 'base'")
        indices = tuple(int(i) for i in out_indices)
        if not indices or len(set(indices)) != len(indices) or any(i not in range(4) for i in indices):
            raise ValueError("out_indices must contain unique stage indices in [0, 3]")
        if indices != tuple(sorted(indices)):
            raise ValueError("out_indices must be in increasing stage order")
        model = create_model(f"visionhope_{arch}", in_chans=in_chans, num_classes=1000, **kwargs)
        self.arch = arch
        self.embed_dims = list(model.embed_dims)
        self.downsample_layers = model.downsample_layers
        self.stages = model.stages
        self.out_norms = nn.ModuleList(LayerNorm2d(d) if out_norm else nn.Identity() for d in self.embed_dims)
        self.out_indices = indices
        self.num_features = [self.embed_dims[i] for i in indices]
        self.channels_last = bool(channels_last)

    def forward(self, x):
        if self.channels_last:
            x = x.contiguous(memory_format=torch.channels_last)
        outs = []
        pending = None
        for i, (down, stage) in enumerate(zip(self.downsample_layers, self.stages)):
            if pending is not None and isinstance(down, Downsample):
                x = down(x, pending)  # the previous stage's last add fused with this input's cast
            else:
                x = down(x if pending is None else x + pending)
            x, pending = HierarchicalVisionHOPE._run_stage(stage, x)
            if i in self.out_indices:
                norm = self.out_norms[i]
                if pending is not None and isinstance(norm, LayerNorm2d):
                    x, y = norm.forward_add(x, pending)
                else:
                    x = x if pending is None else x + pending
                    y = norm(x)
                pending = None
                outs.append(y)
            if i == max(self.out_indices):
                break
        return tuple(outs)


def create_model(name, **kwargs):
    if name not in MODEL_CONFIGS:
        raise ValueError(f"Unknown model {name!r}; choose from {tuple(MODEL_CONFIGS)}")
    config = deepcopy(MODEL_CONFIGS[name])
    config.update(kwargs)
    return HierarchicalVisionHOPE(**config)


def prepare_for_inference(model):
    """Eval mode, fast SRNL inference, LayerScale folded into proj_out / fc2
    (inference/prepare.py:12-54).  Returns preparation counts."""
    blocks = [m for m in model.modules() if isinstance(m, VisionHOPEBlock)]
    model.eval()
    counts = dict(line_mixer=0, srnl=0, operator=0, layernorm2d=0, grn=0, layerscale=0)
    for m in model.modules():
        if isinstance(m, ScanMemories):
            counts["srnl"] += 1
            m.densify()  # read dense by the scan, instead of a copy every call
        elif isinstance(m, ScanMixer):
            counts["operator"] += 1
        elif isinstance(m, LayerNorm2d):
            m.inference_layout = True
            counts["layernorm2d"] += 1
        elif isinstance(m, GlobalResponseNorm):
            counts["grn"] += 1
    for block in blocks:
        for norm in (block.norm1, block.norm2):
            if isinstance(norm, LayerNorm2d):
                norm.emit_autocast_dtype = True  # consumed only by proj_in / fc1
    if isinstance(getattr(model, "norm", None), LayerNorm2d):
        model.norm.emit_autocast_dtype = True  # consumed only by head_pre_logits
    with torch.no_grad():
        for block in blocks:
            counts["line_mixer"] += 1
            for gname, proj in (("gamma1", block.proj_out), ("gamma2", block.ffn.fc2)):
                gamma = getattr(block, gname)
                if gamma is None:
                    continue
                scale = gamma.detach().view(-1).to(dtype=proj.weight.dtype, device=proj.weight.device)
                proj.weight.mul_(scale.view((-1,) + (1,) * (proj.weight.ndim - 1)))
                if proj.bias is not None:
                    proj.bias.mul_(scale)
                setattr(block, gname, None)
                counts["layerscale"] += 1
            block._inference_prepared = True
        for m in model.modules():
            if isinstance(m, PatchEmbedding) or isinstance(m, Downsample):
                counts["batchnorm_folded"] = counts.get("batchnorm_folded", 0) + m.fold_batchnorm()
        for block in blocks:
            for lin in (block.proj_in, block.local_gate, block.operator.W_q, block.proj_out,
                        block.ffn.fc1, block.ffn.fc2):
                if lin is not None:
                    cache_half_weights(lin)
    if blocks:
        model._inference_prepared = True
    return counts
