"""Generate golden vectors from the reference's own CPU code paths (run in the development
container, where the reference tree is importable).

TEST INFRASTRUCTURE.  GRN and LayerNorm2d have CPU implementations in the reference:
``utils/grn.py:26-38`` (grn_reference) and ``models/layers.py:25-35`` (F.layer_norm path of
LayerNorm2d).  This script imports the reference read-only (with a four-alias ``timm`` shim,
timm is not installed), runs those paths on seeded inputs and stores inputs and outputs in
``tests/golden/cpu_*.npz``.

Usage:  python tests/golden/make_golden_cpu.py [--reference <reference checkout>]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VHOPE_REFERENCE"),
                    help="reference checkout (default: the VHOPE_REFERENCE environment variable)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set VHOPE_REFERENCE")
    import oracle.build_ref as br

    br.REF_ROOT = Path(args.reference)
    br._install_reference()
    from visionhope.models.layers import LayerNorm2d
    from visionhope.utils.grn import grn_reference

    manifest = {}
    cases = [("cpu_grn_56x56x96", (4, 96, 14, 14)), ("cpu_grn_7x7x768", (3, 768, 7, 7)),
             ("cpu_ln_96", (4, 96, 14, 14)), ("cpu_ln_768", (3, 768, 7, 7)), ("cpu_ln_64", (2, 64, 9, 9))]
    for i, (name, shape) in enumerate(cases):
        g = torch.Generator().manual_seed(2000 + i)
        B, C, H, W = shape
        x = torch.randn(shape, generator=g)
        if name.startswith("cpu_grn"):
            gamma = torch.randn(1, C, 1, 1, generator=g) * 0.02
            beta = torch.randn(1, C, 1, 1, generator=g) * 0.02
            y = grn_reference(x, gamma, beta, 1e-6)
            arrays = dict(x_nchw=x, gamma=gamma, beta=beta, y_nchw=y)
            fn = "utils/grn.py:grn_reference"
        else:
            ln = LayerNorm2d(C)
            with torch.no_grad():
                ln.weight.copy_(1 + 0.02 * torch.randn(C, generator=g))
                ln.bias.copy_(0.02 * torch.randn(C, generator=g))
            ln.inference_layout = True  # F.layer_norm path (models/layers.py:18-20)
            with torch.no_grad():
                y = ln(x * 3 + 1)
            arrays = dict(x_nchw=x * 3 + 1, weight=ln.weight.detach(), bias=ln.bias.detach(), y_nchw=y)
            fn = "models/layers.py:LayerNorm2d(inference_layout)"
        np.savez_compressed(OUT / f"{name}.npz", **{k: v.detach().float().numpy() for k, v in arrays.items()})
        manifest[name] = dict(fn=fn, shape=list(shape), seed=2000 + i)
    (OUT / "cpu_manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    print("wrote", list(manifest))


if __name__ == "__main__":
    main()
