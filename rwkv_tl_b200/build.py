"""Build ``librwkv_b200.so`` (the C-ABI CUDA library) in-tree for sm_100a.

``python -m rwkv_tl_b200.build`` compiles every ``csrc/*.cu`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and links the
shared library next to this file, where ``rwkv_tl_b200._lib`` loads it. Only
changed sources are recompiled.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "librwkv_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xptxas", "-v" if os.environ.get("RWKV_PTXAS_VERBOSE") else "-O3",
         *os.environ.get("RWKV_B200_NVCC_EXTRA", "").split()]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA library cannot be built")


def _compile(src: Path) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip() and os.environ.get("RWKV_PTXAS_VERBOSE"):
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
