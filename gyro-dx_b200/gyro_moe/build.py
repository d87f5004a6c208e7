"""Builds the sm_100a shared library libgyromoe.so in-tree (nvcc cross-compiles without a GPU).

    python gyro-dx_b200/gyro_moe/build.py [--force]

The library exports the C ABI of include/gyro_moe.h and nothing else; the CUDA runtime is
linked statically so the file loads next to any torch build.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
ROOT = PKG.parents[1]
LIB = PKG / "libgyromoe.so"
SOURCES = ["gx_kernels.cu", "gx_decode_stack.cu", "gx_prefill.cu", "gx_gemm_ts.cu", "gx_router_tc.cu", "gx_ep.cu", "gx_shared.cu", "gx_hc.cu",
           "gx_comm.cu", "gx_abi.cu", "gx_gguf.cpp"]
HEADERS = ["gx_tile.h", "gx_device.cuh", "gx_gemv.cuh", "gx_internal.h", "gx_umma.cuh", "gx_comm.h", "gx_dense.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-cudart", "static", "-I", str(ROOT / "include")]


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "gyro_moe.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    objs = []
    build_dir = PKG.parent / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([NVCC, *ARCH, "-shared", "-cudart", "static", *objs, "-ldl", "-o", str(tmp)], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
