"""Build libqi.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m qweninfer_b200.csrc.build [--verbose]

Produces qweninfer_b200/libqi.so. Sources are compiled in parallel, then linked with
the static CUDA runtime so the library does not depend on which libcudart PyTorch
loaded.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
LIB = PKG / "libqi.so"
SOURCES = ["gemv.cu", "attention.cu", "attention_block.cu", "misc.cu", "norm_rope.cu", "tc_proj.cu", "api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def flags(verbose: bool) -> list[str]:
    f = ["-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(REPO / "include")]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def build(verbose: bool = False, force: bool = False) -> Path:
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [
        REPO / "include" / "qi.h", Path(__file__).resolve()]
    newest = max(p.stat().st_mtime for p in deps)
    if LIB.exists() and not force and LIB.stat().st_mtime >= newest:
        return LIB
    exe = nvcc()

    def compile_one(src: str) -> tuple[str, str]:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [exe, *flags(verbose), "-c", str(CSRC / src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stderr}")
        return str(obj), res.stderr

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    for _, log in results:
        if verbose and log:
            sys.stderr.write(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [exe, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *[o for o, _ in results]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
