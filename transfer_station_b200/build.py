"""Builds the in-tree shared library ``transfer_station_b200/lib/libattn_flash_b200.so``.

CUDA sources are compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``);
the C host layer with gcc. nvcc cross-compiles, so this runs on a machine without a GPU.
Objects go to ``transfer_station_b200/_build`` and are rebuilt when a source or header is
newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
OBJDIR = PKG / "_build"
LIBDIR = PKG / "lib"
LIBNAME = "libattn_flash_b200.so"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]
CC = os.environ.get("CC", "gcc")
CC_FLAGS = ["-O2", "-std=c11", "-fPIC", "-Wall", "-Wextra"]

CU_SOURCES = ["fa_fwd_sm100.cu", "fa_aux.cu", "fa_noalloc.cu", "fa_diag.cu", "fa_peer.cu", "qkv_rope.cu"]
C_SOURCES = ["attn_flash.c", "attn_qkv_rope.c"]


def lib_path() -> Path:
    return LIBDIR / LIBNAME


def _newest_input() -> float:
    files = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.is_file())


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd)}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every CUDA/C source and link the shared library; returns its path."""
    out = lib_path()
    if not force and out.exists() and out.stat().st_mtime >= _newest_input():
        return out
    OBJDIR.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    objs = []
    inc = ["-I", str(INCLUDE), "-I", str(CSRC)]
    for src in CU_SOURCES:
        obj = OBJDIR / (Path(src).stem + ".o")
        extra = ["-Xptxas", "-v"] if ptxas_verbose else []
        _run([NVCC, *ARCH, *NVCC_FLAGS, *extra, *inc, "-c", str(CSRC / src), "-o", str(obj)], verbose or ptxas_verbose)
        objs.append(str(obj))
    for src in C_SOURCES:
        obj = OBJDIR / (Path(src).stem + ".o")
        _run([CC, *CC_FLAGS, *inc, "-c", str(CSRC / src), "-o", str(obj)], verbose)
        objs.append(str(obj))
    tmp = out.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objs, "-lm"], verbose)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(p)
