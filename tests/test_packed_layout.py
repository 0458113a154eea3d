"""The tiled Q6_K, Q5_K, Q3_K and Q2_K layouts and the GEMV's decode arithmetic,
emulated on the CPU (tests/layout_emu.cpp, built here with g++ from the engine's own
packing helpers) and checked against the oracle's matvec with the GEMV parity bar,
max|y - y_ref| <= 2e-4 * max|y_ref|.  A packer or addressing change that the kernel
does not follow fails here without a GPU.
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INC = "/usr/local/cuda/include"


@pytest.fixture(scope="module")
def emu(tmp_path_factory):
    if not shutil.which("g++") or not os.path.exists(os.path.join(CUDA_INC, "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    out = str(tmp_path_factory.mktemp("emu") / "liblayout_emu.so")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", "-I", CUDA_INC, "-I",
                    os.path.join(ROOT, "ramforge_b200", "csrc"), os.path.join(ROOT, "tests", "layout_emu.cpp"),
                    "-o", out], check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    lib.emu_gemv.restype = ctypes.c_int
    lib.emu_gemv.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                             ctypes.c_void_p]
    return lib


def _raw(gtype, M, K, seed):
    if gtype == synth.Q6_K:
        return synth.quantize(gtype, synth.normal(seed, 5, M * K, std=0.02).reshape(M, K))
    return synth.random_blocks(gtype, M, K, seed)


@pytest.mark.parametrize("gtype", [synth.Q6_K, synth.Q5_K, synth.Q3_K, synth.Q2_K])
@pytest.mark.parametrize("M,K", [(1, 256), (65, 512), (130, 768), (200, 4096)])
def test_emulated_gemv_matches_oracle(emu, gtype, M, K):
    raw = np.ascontiguousarray(_raw(gtype, M, K, M + gtype), np.uint8)
    x = synth.normal(9, 7, K, std=1.0)
    y = np.empty(M, np.float32)
    assert emu.emu_gemv(gtype, raw.ctypes.data, M, K, x.ctypes.data, y.ctypes.data) == 0
    ref = orc.matvec(gtype, raw, K, M, x, threads=8)
    assert np.abs(y - ref).max() <= 2e-4 * np.abs(ref).max() + 1e-6
