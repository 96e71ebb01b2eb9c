"""Build libtfb.so (the C-ABI kernel library) in-tree with nvcc for sm_100a.

    python qwen-image21-tensorfold-rtx_b200/build.py [--force] [--verbose]

The library lands next to the Python package (``tfimage/libtfb.so``) so it travels with the source tree; nothing
is installed elsewhere. The build is incremental: objects are rebuilt when their source or a header changed.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
OUT = HERE / "tfimage" / "libtfb.so"
OBJ = HERE / "_build"
SOURCES = ["host.cu", "quant.cu", "fusions.cu", "gemm.cu", "gguf.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr", "-I", str(INCLUDE),
         "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = OBJ / (src + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, newest_header):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lrt"]
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
