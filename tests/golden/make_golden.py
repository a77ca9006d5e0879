"""Generate golden vectors from the reference's own CUDA kernels (run on a B200).

TEST INFRASTRUCTURE.  The reference ships no golden vectors and has no CPU path for SRNL,
so these fixtures are produced by the reference's own extensions, compiled from its
sources by ``oracle/build_ref.py`` into ``oracle/_ref/`` (built in the development
container, shipped to the GPU box with the snapshot).  Each case stores its inputs and the
reference output in float32 (bf16/fp16 inputs are widened exactly) in ``tests/golden/``.

Usage (GPU box):  python tests/golden/make_golden.py [--out DIR]

Every buffer the reference kernels write is allocated with exactly the shapes the reference
allocates (models/srnl_core/chunk.py:219-231, 421-435; lines.py:240-255, 478-495).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.build_ref import load_built  # noqa: E402

OUT = Path(__file__).resolve().parent
DEV = torch.device("cuda:0")


def mems(gen, dirs, heads, D, kind):
    if kind == "default":
        mats = [np.clip(gen.normal(0, 0.01, (dirs, heads, D, D)), -0.02, 0.02) for _ in range(3)]
        vecs = [np.zeros((dirs, heads, D)) for _ in range(2)]
    else:  # stress: data-dependent gates, clamps exercised
        mats = [gen.normal(0, 0.35, (dirs, heads, D, D)) for _ in range(3)]
        vecs = [gen.normal(0, 0.6, (dirs, heads, D)), gen.normal(-1.0, 1.2, (dirs, heads, D))]
    return [torch.tensor(np.asarray(a, np.float32), device=DEV) for a in (*mats, *vecs)]


def f32np(t):
    return t.detach().float().cpu().numpy()


def serialize(img):
    B, H, W, C = img.shape
    hw = img.reshape(B, H * W, C)
    wh = img.transpose(1, 2).reshape(B, H * W, C)
    return torch.stack([hw, hw.flip(1), wh, wh.flip(1)], dim=1).contiguous()


def case_fused(name, gen, B, H, W, heads, D, dtype, kind, per_dir):
    ext = load_built("vhref_fused_bf16" if dtype == torch.bfloat16 else "vhref_fused_fp32")
    C = heads * D
    M = mems(gen, 4, heads, D, kind)
    img = torch.tensor(gen.normal(size=(B, H, W, C)), dtype=dtype, device=DEV)
    qimg = torch.tensor(gen.normal(size=(B, H, W, C)), dtype=dtype, device=DEV)
    xs, qs = serialize(img), serialize(qimg)
    skip = torch.tensor(gen.normal(0, 0.5, size=(4 * C,) if per_dir else (C,)), dtype=torch.float32, device=DEV)
    wts = torch.tensor(gen.normal(1.0, 0.3, size=(4, C)), dtype=torch.float32, device=DEV)
    out = ext.srnl_line_forward_seq_noatomic(*M, xs, qs, skip, wts, H, W, D)
    return dict(kind="spatial", fn="srnl_line_forward_seq_noatomic", H=H, W=W, D=D,
                io=str(dtype)), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                     xs=xs, qs=qs, skip=skip, weight=wts, out=out)


def case_sequence(name, gen, B, R, heads, L, D, chunks, dtype, kind):
    ext = load_built("vhref_fused_bf16" if dtype == torch.bfloat16 else "vhref_fused_fp32")
    C = heads * D
    M = mems(gen, R, heads, D, kind)
    x = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=dtype, device=DEV)
    q = torch.tensor(gen.normal(size=(B, R, L, C)), dtype=dtype, device=DEV)
    y = ext.srnl_sequence_forward(*M, x, q, list(chunks))
    return dict(kind="sequence", fn="srnl_sequence_forward", chunks=list(chunks), q_mode="raw",
                io=str(dtype)), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                     x=x, q=q, y=y)


def _chunk_buffers(n_flat, L, D, num_chunks):
    f = dict(device=DEV, dtype=torch.float32)
    return [torch.empty((n_flat, max(num_chunks - 1, 0), D, D), **f),
            torch.empty((n_flat, L, D), **f), torch.empty((n_flat, L, D), **f),
            *[torch.empty((n_flat, L), **f) for _ in range(5)]]


def case_chunk_normalized(name, gen, B, R, heads, L, D, chunk, dtype, kind):
    """srnl_forward with fp32 unit queries (ordinary path, chunk.py:172-284); L % chunk == 0."""
    assert L % chunk == 0
    ext = load_built("vhref_chunk_bf16" if dtype == torch.bfloat16 else "vhref_chunk_fp32")
    M = mems(gen, R, heads, D, kind)
    x = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=dtype, device=DEV)
    q = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=torch.float32, device=DEV)
    q = (q / q.norm(dim=-1, keepdim=True)).contiguous()
    n_flat, state_count = B * R * heads, R * heads
    Ms = [m.contiguous().view(state_count, D, D) for m in M[:3]] + [m.contiguous().view(state_count, D) for m in M[3:]]
    bufs = _chunk_buffers(n_flat, L, D, L // chunk)
    one = torch.empty((1,), device=DEV, dtype=torch.float32)
    y = ext.srnl_forward(*Ms, x.view(n_flat, L, D), q.view(n_flat, L, D), *bufs, one, one.clone(),
                         chunk, D, state_count, 0)
    return dict(kind="sequence", fn="srnl_forward", chunks=[chunk] * R, q_mode="norm",
                io=str(dtype)), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                     x=x, q=q, y=y.view(B, R, heads, L, D))


def case_chunk_qraw(name, gen, B, heads, L, D, chunk, dtype, kind):
    """srnl_forward_qraw (4 directions, raw queries, chunk.py:366-505); L % chunk == 0."""
    assert L % chunk == 0
    ext = load_built("vhref_chunk_bf16" if dtype == torch.bfloat16 else "vhref_chunk_fp32")
    R, C = 4, heads * D
    M = mems(gen, R, heads, D, kind)
    x = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=dtype, device=DEV)
    q = torch.tensor(gen.normal(size=(B, R, L, C)), dtype=dtype, device=DEV)
    n_flat, state_count = B * R * heads, R * heads
    Ms = [m.contiguous().view(state_count, D, D) for m in M[:3]] + [m.contiguous().view(state_count, D) for m in M[3:]]
    bufs = _chunk_buffers(n_flat, L, D, L // chunk)
    one = torch.empty((1,), device=DEV, dtype=torch.float32)
    qinv = torch.empty((n_flat, L), device=DEV, dtype=torch.float32)
    y = ext.srnl_forward_qraw(*Ms, x.view(n_flat, L, D), q, *bufs, one, one.clone(), qinv, chunk, D,
                              state_count, 0, heads, 1)
    return dict(kind="sequence", fn="srnl_forward_qraw", chunks=[chunk] * R, q_mode="raw",
                io=str(dtype)), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                     x=x, q=q, y=y.view(B, R, heads, L, D))


def case_varline(name, gen, B, heads, H, W, D, kind):
    """srnl_forward_qraw_varline (bf16, lines.py:402-560): row chunk W, column chunk H."""
    ext = load_built("vhref_lines_bf16")
    R, C, L = 4, heads * D, H * W
    M = mems(gen, R, heads, D, kind)
    x = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=torch.bfloat16, device=DEV)
    q = torch.tensor(gen.normal(size=(B, R, L, C)), dtype=torch.bfloat16, device=DEV)
    n_flat, state_count = B * R * heads, R * heads
    row_nc, col_nc = L // W, L // H
    max_nc, max_cs = max(row_nc, col_nc), max(W, H)
    max_sub = (max_cs + 7) // 8
    groups = B * heads
    packed_nc = groups * (2 * row_nc + 2 * col_nc)
    packed_pc = groups * (2 * max(row_nc - 1, 0) + 2 * max(col_nc - 1, 0))
    f = dict(device=DEV, dtype=torch.float32)
    Ms = [m.contiguous().view(state_count, D, D) for m in M[:3]] + [m.contiguous().view(state_count, D) for m in M[3:]]
    y = ext.srnl_forward_qraw_varline(
        *Ms, x.view(n_flat, L, D), q, torch.empty((max(packed_pc, 1), D, D), **f),
        torch.empty((n_flat, L, D), **f), torch.empty((n_flat, L, D), **f),
        *[torch.empty((n_flat, L), **f) for _ in range(6)],
        torch.empty((packed_nc * max_sub, D, D), **f), torch.empty((packed_nc, D, D), **f),
        W, H, D, state_count, heads, 1, max_nc, max_sub)
    return dict(kind="sequence", fn="srnl_forward_qraw_varline", chunks=[W, W, H, H], q_mode="raw",
                io="torch.bfloat16"), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                           x=x, q=q, y=y.view(B, R, heads, L, D))


def case_large(name, gen, B, R, heads, L, D, chunk, kind):
    """srnl_forward_qraw_large (bf16, chunk > 64, lines.py:183-311) with tail padding applied."""
    ext = load_built("vhref_lines_bf16")
    C = heads * D
    M = mems(gen, R, heads, D, kind)
    x = torch.tensor(gen.normal(size=(B, R, heads, L, D)), dtype=torch.bfloat16, device=DEV)
    q = torch.tensor(gen.normal(size=(B, R, L, C)), dtype=torch.bfloat16, device=DEV)
    pad = (chunk - L % chunk) % chunk
    xp = torch.nn.functional.pad(x, (0, 0, 0, pad)).contiguous()
    qp = torch.nn.functional.pad(q, (0, 0, 0, pad)).contiguous()
    Lp = L + pad
    n_flat, state_count = B * R * heads, R * heads
    nc, max_sub = Lp // chunk, (chunk + 7) // 8
    f = dict(device=DEV, dtype=torch.float32)
    Ms = [m.contiguous().view(state_count, D, D) for m in M[:3]] + [m.contiguous().view(state_count, D) for m in M[3:]]
    y = ext.srnl_forward_qraw_large(
        *Ms, xp.view(n_flat, Lp, D), qp, torch.empty((n_flat, max(nc - 1, 0), D, D), **f),
        torch.empty((n_flat, Lp, D), **f), torch.empty((n_flat, Lp, D), **f),
        *[torch.empty((n_flat, Lp), **f) for _ in range(6)],
        torch.empty((n_flat, nc * max_sub, D, D), **f), torch.empty((n_flat, nc, D, D), **f),
        chunk, D, state_count, heads, 1, max_sub)
    y = y.view(B, R, heads, Lp, D)[:, :, :, :L]
    return dict(kind="sequence", fn="srnl_forward_qraw_large", chunks=[chunk] * R, q_mode="raw",
                io="torch.bfloat16"), dict(M_m=M[0], M_v=M[1], M_k=M[2], M_eta=M[3], M_alpha=M[4],
                                           x=x, q=q, y=y)


def case_qnorm(name, gen, B, L, heads, D, dtype):
    ext = load_built("vhref_qnorm_bf16" if dtype == torch.bfloat16 else "vhref_qnorm_fp32")
    q = torch.tensor(gen.normal(size=(B, 4, L, heads * D)), dtype=dtype, device=DEV)
    out, inv = ext.visionhope_qnorm_forward(q, heads, D, True)
    return dict(kind="qnorm", heads=heads, D=D, io=str(dtype)), dict(q=q, out=out, inv=inv)


def case_dirfuse(name, gen, B, heads, H, W, D, dtype, channels_last, per_dir):
    ext = load_built("vhref_dirfuse_bf16" if dtype == torch.bfloat16 else "vhref_dirfuse_fp32")
    L, C = H * W, heads * D
    y = torch.tensor(gen.normal(size=(B, 4, heads, L, D)), dtype=dtype, device=DEV)
    x = torch.tensor(gen.normal(size=(B, 4, heads, L, D)), dtype=dtype, device=DEV)
    skip = torch.tensor(gen.normal(size=(4, heads, D) if per_dir else (heads, D)), dtype=torch.float32, device=DEV)
    scale = torch.tensor(gen.normal(1, 0.3, size=(4, C)), dtype=torch.float32, device=DEV)
    out = ext.visionhope_postprocess_scale_forward(y, x, skip, scale, H, W, channels_last, False)
    return dict(kind="dirfuse", H=H, W=W, channels_last=channels_last, io=str(dtype)), dict(
        y=y, x=x, skip=skip, scale=scale, out=out.contiguous())


def case_grn(name, gen, B, H, W, C, dtype):
    ext = load_built("vhref_grn")
    x = torch.tensor(gen.normal(size=(B, H, W, C)), dtype=dtype, device=DEV).permute(0, 3, 1, 2)
    gamma = torch.tensor(gen.normal(0, 0.02, size=(1, C, 1, 1)), dtype=torch.float32, device=DEV)
    beta = torch.tensor(gen.normal(0, 0.02, size=(1, C, 1, 1)), dtype=torch.float32, device=DEV)
    y = torch.empty_like(x, dtype=torch.float32, memory_format=torch.channels_last)
    gx = torch.empty((B, C), device=DEV, dtype=torch.float32)
    inv = torch.empty((B,), device=DEV, dtype=torch.float32)
    ext.grn_forward_cuda(x, gamma, beta, y, gx, inv, 1e-6)
    return dict(kind="grn", io=str(dtype)), dict(x_nhwc=x.permute(0, 2, 3, 1).contiguous(), gamma=gamma,
                                                 beta=beta, y_nhwc=y.permute(0, 2, 3, 1).contiguous(),
                                                 gx=gx, inv_den=inv)


CASES = [
    ("spatial_bf16_default", case_fused, (2, 8, 8, 2, 16, torch.bfloat16, "default", False)),
    ("spatial_bf16_stress_rect", case_fused, (2, 7, 9, 2, 16, torch.bfloat16, "stress", False)),
    ("spatial_fp32_stress_perdir", case_fused, (1, 6, 10, 3, 16, torch.float32, "stress", True)),
    ("spatial_bf16_stress_d8", case_fused, (1, 5, 6, 2, 8, torch.bfloat16, "stress", False)),
    ("sequence_bf16_stress", case_sequence, (2, 4, 2, 30, 16, (6, 6, 5, 5), torch.bfloat16, "stress")),
    ("sequence_fp32_pad", case_sequence, (1, 2, 2, 29, 16, (8, 8), torch.float32, "stress")),
    ("chunk_norm_fp32_cfg1", case_chunk_normalized, (2, 1, 4, 196, 16, 14, torch.float32, "default")),
    ("chunk_norm_fp32_stress", case_chunk_normalized, (2, 1, 4, 196, 16, 14, torch.float32, "stress")),
    ("chunk_qraw_bf16_stress", case_chunk_qraw, (1, 2, 36, 16, 6, torch.bfloat16, "stress")),
    ("varline_bf16_stress", case_varline, (1, 2, 5, 8, 16, "stress")),
    ("large_bf16_stress", case_large, (1, 2, 1, 150, 16, 70, "stress")),
    ("qnorm_bf16", case_qnorm, (2, 20, 3, 16, torch.bfloat16)),
    ("dirfuse_fp32_cl", case_dirfuse, (2, 2, 5, 7, 16, torch.float32, True, False)),
    ("dirfuse_bf16_nchw_perdir", case_dirfuse, (1, 2, 6, 4, 16, torch.bfloat16, False, True)),
    ("grn_fp32", case_grn, (2, 7, 7, 96, torch.float32)),
    ("grn_bf16", case_grn, (2, 5, 5, 64, torch.bfloat16)),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(OUT))
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    manifest = {}
    for i, (name, fn, params) in enumerate(CASES):
        gen = np.random.default_rng(1000 + i)
        meta, arrays = fn(name, gen, *params)
        torch.cuda.synchronize()
        np.savez_compressed(out / f"{name}.npz", **{k: f32np(v) for k, v in arrays.items()})
        meta.update(seed=1000 + i, params=[str(p) for p in params])
        manifest[name] = meta
        print("wrote", name, flush=True)
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
