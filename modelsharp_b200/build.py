"""Builds libms_cuda_nbits.so in-tree for sm_100a with nvcc (no JIT cache, no torch types).

    python -m modelsharp_b200.build
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libms_cuda_nbits.so"
SOURCES = ["msq_api.cu", "msq_repack.cu", "msq_generic.cu", "msq_gemv.cu", "msq_gemv_mma.cu", "msq_gemm.cu",
           "msq_noalloc.cu", "msq_decoder.cu", "msq_gemv_tc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libms_cuda_nbits.so")
    return cand


def needs_rebuild() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "ms_cuda_nbits.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every translation unit in parallel into _build/ and links the shared library."""
    if not force and not needs_rebuild():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    obj_dir = PKG / "_build"
    obj_dir.mkdir(exist_ok=True)
    flags = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC"]

    def compile_one(src: str) -> Path:
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *flags, "-c", "-o", str(obj), str(CSRC / src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src} ({r.returncode}):\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
