"""GPU parity of the tensor-core batched GEMM (rf_qgemm) and of the batched
prompt path against the CPU oracle (the reference's token-by-token executor).

Tolerance of the GEMM: max|y - y_ref| <= 2e-4 * max|y_ref| + 1e-6 per token, the
GEMV bar; the operands are split into bf16 hi + lo (three products), which keeps
the error near 2^-16 of the reference's f32 products.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import QMatrix, synth
from ramforge_b200 import _lib

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)


def _weights(gtype, M, K, seed):
    return synth.quantize(gtype, synth.normal(seed, 100 + gtype, M * K, std=0.02).reshape(M, K))


def _qgemm(gtype, M, K, T, seed=1):
    import torch
    raw = _weights(gtype, M, K, seed)
    x = synth.normal(seed, 9, T * K, std=1.0).reshape(T, K)
    m = QMatrix(gtype, raw, M, K)
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((T, M), float("nan"), device="cuda")
    m.gemm(dx.data_ptr(), dy.data_ptr(), T)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    w = _lib.ctypes.c_uint32()
    _lib.check(_lib.lib().rf_qgemm_error_word(_lib.ctypes.byref(w)))
    assert w.value == 0
    m.close()
    return raw, x, y


@pytest.mark.parametrize("gtype", [synth.Q4_K, synth.Q8_0])
@pytest.mark.parametrize("M,K,T", [(64, 256, 1), (130, 512, 7), (384, 1024, 128), (300, 768, 129),
                                   (4096, 4096, 200)])
def test_qgemm_matches_reference_matvec_per_token(gtype, M, K, T):
    raw, x, y = _qgemm(gtype, M, K, T)
    assert not np.isnan(y).any()
    worst = 0.0
    for t in range(T):
        ref = orc.matvec(gtype, raw, K, M, x[t], threads=THREADS)
        err = np.abs(y[t] - ref).max() / (np.abs(ref).max() + 1e-30)
        worst = max(worst, err)
        assert np.abs(y[t] - ref).max() <= 2e-4 * np.abs(ref).max() + 1e-6, (gtype, M, K, T, t, err)
    print(f"qgemm {gtype} {M}x{K} T={T}: worst relative error {worst:.2e}")


def test_qgemm_refuses_unsupported_formats():
    import torch
    raw = _weights(synth.Q4_0, 64, 256, 2)
    m = QMatrix(synth.Q4_0, raw, 64, 256)
    dx = torch.zeros(4, 256, device="cuda")
    dy = torch.zeros(4, 64, device="cuda")
    rc = _lib.lib().rf_qgemm(m._h, dx.data_ptr(), dy.data_ptr(), 4, None)
    assert rc == _lib.RF_EUNSUPPORTED
    m.close()
