"""Builds libxvec_gpu.so in-tree with nvcc for sm_100a (no JIT, no torch)."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libxvec_gpu.so")
SOURCES = ["capi.cu", "flat_kernels.cu", "flat_tc.cu", "index_quantized.cu", "merge.cu", "noalloc.cu", "sq8.cu", "ivfpq.cu", "rabitq.cu", "refine_api.cu", "kmeans.cu", "ivf_flat.cu", "ivf_file.cu", "pq_train.cu", "comm.cu", "flat_stream.cu", "rotation.cu", "diskann.cu"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "xvec_gpu.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs, procs = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if _stale(obj, path):
            cmd = [NVCC, *FLAGS, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                                stderr=subprocess.STDOUT, text=True)))
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{out}")
        if verbose and out.strip():
            print(out)
    if procs or not os.path.exists(LIB):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB,
               "-cudart", "static", "-ldl"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
