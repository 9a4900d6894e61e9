"""Build recipe for libheadshot_cuda.so (sm_100a) — run in place.

`python -m headshot_b200.build` compiles every file in headshot_b200/csrc
with nvcc into headshot_b200/libheadshot_cuda.so.  Objects go to
headshot_b200/_build/.  Nothing is JIT-compiled at import time: the built
library travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libheadshot_cuda.so"
BUILD = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-I" + str(PKG.parent / "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libheadshot_cuda.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *(PKG.parent / "include").glob("*.h"), Path(__file__)]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if not force and not ptxas_info and not _stale(obj, src):
            continue
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or ptxas_info or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv, force="--force" in sys.argv)
