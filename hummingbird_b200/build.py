"""Build `hummingbird_b200/libhb_b200.so` in-tree with nvcc for sm_100a.

    python -m hummingbird_b200.build [--verbose]

One shared library, relocatable device code (the kernels share one device status word), static cudart,
no torch types anywhere in the ABI.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libhb_b200.so"
SOURCES = ["abi.cu", "attn_kernel.cu", "dense_attn.cu", "band_attn.cu", "band_fused.cu", "w8a8.cu", "dit_glue.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build hummingbird_b200")
    return cand


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "hb_b200.h"]
    if LIB.exists() and not force and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-shared", "-Xcompiler", "-fPIC",
           "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, srcs)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout, res.stderr, sep="\n")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print(LIB)
