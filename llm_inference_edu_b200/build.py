"""Builds libqwen_b200.so in-tree with nvcc for sm_100a.

    python -m llm_inference_edu_b200.build

The library links the CUDA runtime statically, so loading it needs no GPU
and no driver; only calls that touch the device do.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libqwen_b200.so")
SOURCES = ["ops.cu", "decode.cu", "prefill.cu", "tc_gemm.cu", "tp.cu", "sampling.cu", "runtime.cu", "static_scratch.cu", "synthetic.cpp", "loader.cpp", "bridge.cpp", "tokenizer.cpp"]
HEADERS = ["common.cuh", "decode.cuh", "prefill.cuh", "multitoken.cuh", "tc_gemm.cuh", "tp.cuh", "sampling.cuh", "json.h", "unicode_tables.inc"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # Separate roundings for a*b+c unless fmaf() is written explicitly, so the
    # elementwise arithmetic rounds like the reference's f32 expressions.
    "-fmad=false",
    "--cudart", "static",
    "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off",
]


def _stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "qwen_b200.h"))
    deps.append(os.path.join(os.path.dirname(HERE), "include", "qwen_b200_bridge.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    # An object is rebuilt when its source, or any shared header, is newer.
    hdrs = [os.path.join(CSRC, f) for f in HEADERS]
    hdrs.append(os.path.join(os.path.dirname(HERE), "include", "qwen_b200.h"))
    hdrs.append(os.path.join(os.path.dirname(HERE), "include", "qwen_b200_bridge.h"))
    t_hdr = max(os.path.getmtime(h) for h in hdrs)
    objs, procs = [], []
    for src in SOURCES:
        obj = os.path.join(objdir, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        path = os.path.join(CSRC, src)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) > max(t_hdr, os.path.getmtime(path)):
            continue
        cmd = ["nvcc", *NVCC_FLAGS, "-c", path, "-o", obj]
        if src.endswith(".cpp"):
            cmd = ["nvcc", "-x", "cu", *NVCC_FLAGS, "-c", path, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((cmd, subprocess.Popen(cmd)))
    for cmd, proc in procs:
        if proc.wait() != 0:
            raise subprocess.CalledProcessError(proc.returncode, cmd)
    tmp = OUT + ".tmp"
    cmd = ["nvcc", "-shared", "--cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
           *objs, "-o", tmp, "-Xcompiler", "-fopenmp", "-lgomp"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(OUT)
