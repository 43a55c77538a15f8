"""Build libmllm_cuda.so in-tree for sm_100a with nvcc (no torch extension machinery).

The library exports the C ABI of include/mllm.h.  Objects go to microllm-lab_b200/_build/; the shared
library lands next to this file so that it travels with the source tree.

``build(timeline=True)`` (``python microllm-lab_b200/build.py --timeline``) also links
libmllm_cuda_timeline.so: the same objects except cdec.cu, compiled with -DMLLM_CDEC_TIMELINE so that
the cluster decode kernel stores a globaltimer stamp at every stage boundary of one forward
(``bench.py --case timeline`` reads them).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libmllm_cuda.so")
OUT_TIMELINE = os.path.join(HERE, "libmllm_cuda_timeline.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v"]
if os.environ.get("MLLM_FAST_BUILD"):  # development: only the PetitGPT-shape instantiation
    CUFLAGS += ["-DMLLM_FAST_BUILD"]
SOURCES = ["engine.cu", "decode.cu", "decode1.cu", "cdec.cu", "gemv.cu", "gemv_dense.cu", "gemm.cu", "gemm_tc5.cu", "lwe.cu",
           "pgw.cpp"]
HEADERS = ["cdec.cuh", "device_common.cuh", "engine.cuh", "lwe.cuh", "pgw.hpp", "q4mma.cuh", "tc5.cuh"]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, timeline: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "mllm.h")]
    # objects built with other flags (e.g. MLLM_FAST_BUILD) are rebuilt
    stamp = os.path.join(BUILD, "flags.txt")
    flags = " ".join([NVCC, *ARCH, *CUFLAGS])
    if not os.path.exists(stamp) or open(stamp).read() != flags:
        for f in os.listdir(BUILD):
            if f.endswith(".o"):
                os.remove(os.path.join(BUILD, f))
        with open(stamp, "w") as fh:
            fh.write(flags)
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            if src.endswith(".cu"):
                cmd = [NVCC, *ARCH, *CUFLAGS, "-c", s, "-o", o]
            else:
                cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-c", s, "-o", o]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError(f"compile failed: {src}")
            with open(o + ".log", "w") as f:
                f.write(r.stdout + r.stderr)
    if _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    if timeline:
        s = os.path.join(CSRC, "cdec.cu")
        o = os.path.join(BUILD, "cdec_timeline.cu.o")
        if _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, *CUFLAGS, "-DMLLM_CDEC_TIMELINE", "-c", s, "-o", o]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError("compile failed: cdec.cu (timeline)")
        tobjs = [o if x.endswith("cdec.cu.o") else x for x in objs]
        if _stale(OUT_TIMELINE, tobjs):
            cmd = [NVCC, *ARCH, "-shared", "-o", OUT_TIMELINE, *tobjs, "-lcudart"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError("link failed (timeline)")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, timeline="--timeline" in sys.argv))
