"""Build `hummingbird_b200/libhb_b200.so` in-tree with nvcc for sm_100a.

    python -m hummingbird_b200.build [--verbose]

Two shared libraries, static cudart, no torch types anywhere in the ABI:
  libhb_b200.so  the kernels (relocatable device code: they share one device status word);
  libhb_comm.so  the NCCL exchanges of the multi-GPU paths (include/hb_comm.h), linked with libnccl.so.2.
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
COMM_LIB = PKG / "libhb_comm.so"
COMM_SOURCES = ["comm.cu"]
SOURCES = ["abi.cu", "attn_kernel.cu", "attn_dense.cu", "dense_attn.cu", "band_attn.cu", "cross_attn.cu", "w8a8.cu",
           "dit_glue.cu"]
# Compiled as whole-program device code (no -rdc) into an object linked into the same library: ptxas ignores
# setmaxnreg in relocatable device code, and these kernels rebalance registers between warpgroups with it.
WHOLE_PROGRAM_SOURCES = ["band_fused.cu", "band_proj.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build hummingbird_b200")
    return cand


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    wp_srcs = [CSRC / s for s in WHOLE_PROGRAM_SOURCES]
    deps = srcs + wp_srcs + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "hb_b200.h"]
    if LIB.exists() and not force and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    common = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I",
              str(ROOT / "include")]
    if verbose:
        common.insert(0, "-Xptxas=-v")

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(res.stdout, res.stderr, sep="\n")

    objs = []
    for src in wp_srcs:
        obj = LIB.parent / (src.stem + ".wp.o")
        run([nvcc(), *common, "-c", "-o", str(obj), str(src)])
        objs.append(obj)
    tmp = LIB.with_suffix(".so.tmp")
    try:
        run([nvcc(), *common, "-rdc=true", "-shared", "-o", str(tmp), *map(str, srcs), *map(str, objs)])
    finally:
        for obj in objs:
            obj.unlink(missing_ok=True)
    os.replace(tmp, LIB)
    return LIB


def build_comm(force: bool = False) -> Path:
    """The NCCL exchange library (needs the NCCL headers and libnccl.so.2 of the CUDA image)."""
    srcs = [CSRC / s for s in COMM_SOURCES]
    deps = srcs + [CSRC / "hb_status.h", ROOT / "include" / "hb_comm.h"]
    if COMM_LIB.exists() and not force and all(COMM_LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return COMM_LIB
    tmp = COMM_LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I",
           str(ROOT / "include"), "-o", str(tmp), *map(str, srcs), "-lnccl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, COMM_LIB)
    return COMM_LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    build_comm(force="--force" in sys.argv)
    print(LIB)
    print(COMM_LIB)
