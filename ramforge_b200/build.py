"""Builds the native libraries in-tree (they travel with the source tree).

  ramforge_b200/librfcuda.so   decode engine: sm_100a kernels + C ABI (include/rfcuda.h)
  ramforge_b200/librfsynth.so  seeded synthetic GGUF models / GGUF block encoders (host only)

Run as `python -m ramforge_b200.build` or through __graft_entry__.build().
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2,-ffp-contract=off", "--expt-relaxed-constexpr",
                     "-I" + os.path.join(ROOT, "include")]
CUDA_SOURCES = ["rf_kernels.cu", "rf_gemv.cu", "rf_prefill.cu", "rf_allreduce.cu", "rf_engine.cu", "rf_ops.cu",
                "rf_common.cpp"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_synth(force=False) -> str:
    out = os.path.join(PKG, "librfsynth.so")
    src = os.path.join(CSRC, "rfsynth.cpp")
    if force or _newer(out, [src, os.path.join(CSRC, "rfsynth.h")]):
        _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-pthread", "-o", out, src])
    return out


def build_cuda(force=False, verbose_ptxas=False) -> str:
    out = os.path.join(PKG, "librfcuda.so")
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "rfcuda.h"))
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES]
    if not (force or _newer(out, srcs + headers)):
        return out
    os.makedirs(BUILD, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if force or _newer(obj, [src] + headers):
            flags = list(NVCC_FLAGS)
            if verbose_ptxas and src.endswith(".cu"):
                flags += ["-Xptxas", "-v"]
            r = _run([NVCC] + flags + ["-c", src, "-o", obj])
            if verbose_ptxas:
                sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(compile_one, srcs))
    _run([NVCC] + ARCH + ["-shared", "-o", out] + objs + ["-ldl", "-lpthread"])
    return out


def build_all(force=False) -> None:
    build_synth(force)
    build_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", os.path.join(PKG, "librfcuda.so"), os.path.join(PKG, "librfsynth.so"))
