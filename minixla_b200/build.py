"""Builds libminixla_b200.so in-tree with nvcc for sm_100a.

Run as ``python -m minixla_b200.build`` (or through ``__graft_entry__.build()``).
nvcc cross-compiles on machines without a GPU.  The result lands in
``minixla_b200/_lib/`` so it ships with the source tree.
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
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libminixla_b200.so"
SOURCES = ["runtime.cu", "graph_plan.cu", "gemm_launch.cu", "exec_graph.cu", "exec_streamed.cu", "exec_sharded.cu",
           "fused_gemm.cu", "fused_gemm_pair.cu", "fused_gemm_pair3.cu", "elementwise.cu", "skinny_gemm.cu", "noalloc.cu", "hostcopy.cu", "peer_ipc.cu", "tensor_maps.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build minixla_b200")
    return exe


def build_lib(verbose: bool = False, extra: list[str] | None = None) -> Path:
    LIB_DIR.mkdir(exist_ok=True)
    objs = []
    common = [
        "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden",
        "-I", str(ROOT / "include"), "--expt-relaxed-constexpr", *(extra or []),
    ]
    for src in SOURCES:
        obj = LIB_DIR / (Path(src).stem + ".o")
        cmd = [nvcc(), *common, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs, "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        Path(o).unlink(missing_ok=True)
    return LIB


if __name__ == "__main__":
    print(build_lib(verbose="-v" in sys.argv))
