"""Build the sm_100a library in-tree: tinyminigo_b200/lib/libtmg_cuda.so.

nvcc compiles each translation unit for `-gencode arch=compute_100a,
code=sm_100a` (cross-compiles without a GPU), in parallel, then links one
shared library with the static CUDA runtime.  Rebuilds only what changed.

    python -m tinyminigo_b200.build [--force] [-v]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INC = PKG.parent / "include"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libtmg_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-I", str(CSRC), "-I", str(INC)]
SOURCES = ["api.cu", "gemv.cu", "attn.cu", "prefill.cu", "sample.cu", "tp.cu", "gemm_sm100.cu",
           "decode_fused.cu", "decode_fused_group.cu", "attn_noalloc.cu", "gemv_i8.cu", "attn_tma.cu", "attn_prefill_tc.cu",
           "loader.cpp", "rng.cpp"]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return p


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INC.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, force: bool, hmt: float) -> Path:
    obj = OBJ / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hmt):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *NVCC_FLAGS, "-x", "c++", "-c", str(src), "-o", str(obj)]
    if verbose and src.suffix == ".cu":
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    hmt = _headers_mtime()
    srcs = [CSRC / s for s in SOURCES]
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, force, hmt), srcs))
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
