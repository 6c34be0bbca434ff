"""Build recipe for liblighthouse_b200.so (sm_100a only).

Compiles every ``csrc/*.cu`` with nvcc for ``arch=compute_100a,code=sm_100a``
into objects under ``_build/`` and links them into
``liblighthouse_b200.so`` next to this file (in-tree, so the library travels
with the repository snapshot).  Rebuilds only what changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "liblighthouse_b200.so"
INCLUDE = PKG.parent / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE)]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: pathlib.Path, verbose: bool) -> pathlib.Path:
    obj = OBJ / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> pathlib.Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        subprocess.run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"], check=True)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(verbose="-v" in sys.argv))
