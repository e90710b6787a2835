"""Build libh3b200.so (the C-ABI library of the sm_100a kernels) in-tree.

    python minimax-h3-tensorfold-rtx_b200/build.py [--force] [--verbose] [--define NAME=VALUE ...] [--out PATH]

nvcc cross-compiles for sm_100a without a GPU.  The output lands in
minimax-h3-tensorfold-rtx_b200/tfvideo/_native/libh3b200.so, next to the Python package that loads it.  --define
and --out build a variant elsewhere (e.g. --define H3_GEMM_PAIR=1 for the CTA-pair GEMM), which tfvideo.native loads
when the H3B200_LIB environment variable names it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OUT = PKG / "tfvideo" / "_native" / "libh3b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA 12.9 toolkit expected)")
    return cand


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "h3b200.h"]


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False, defines: tuple[str, ...] = (), out: Path | None = None) -> Path:
    target = Path(out) if out else OUT
    if not force and not defines and out is None and not stale():
        return OUT
    target.parent.mkdir(parents=True, exist_ok=True)
    tmp = target.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2",
           f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr", "-Xptxas", "-v" if verbose else "-O3",
           *[f"-D{d}" for d in defines], "-o", str(tmp), str(CSRC / "h3b200.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libh3b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--define", action="append", default=[], help="NAME=VALUE passed to nvcc as -DNAME=VALUE")
    ap.add_argument("--out", default=None, help="write the library here instead of tfvideo/_native")
    a = ap.parse_args()
    print(build(a.force, a.verbose, tuple(a.define), a.out))
