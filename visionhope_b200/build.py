"""Build recipe for libvhope.so (sm_100a), the C-ABI library behind ``visionhope_b200``.

Each ``csrc/*.cu`` translation unit is compiled in parallel with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked into
``visionhope_b200/libvhope.so`` (in-tree, so it travels with the repository snapshot).
The library depends only on the CUDA runtime (linked statically by nvcc).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ_DIR = PKG / "_build"
LIB = PKG / "libvhope.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise FileNotFoundError("nvcc not found")
    return cand


def _flags(verbose: bool):
    f = ["-O3", "-lineinfo", "-std=c++17", *ARCH, "-Xcompiler", "-fPIC,-O2",
         f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr"]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return [*CSRC.glob("*.cu"), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h"),
            Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def _compile(src: Path, verbose: bool):
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc(), *_flags(verbose), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel for sm_100a and link libvhope.so (skipped when up to date)."""
    if not force and not verbose and up_to_date():
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if verbose:
        for (obj, log) in results:
            sys.stderr.write(f"== {obj.name}\n{log}")
    tmp = LIB.with_name(f".libvhope.{os.getpid()}.so")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(o) for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose="-v" in sys.argv))
