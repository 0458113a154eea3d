"""rf_decode_attention_noalloc: decode attention for callers that cannot call
cudaMalloc (their device memory belongs to another allocator's pool, or they
cannot afford the device synchronisation an allocation may imply).  Its split-K
scratch is a fixed 16 MiB array inside librfcuda.so instead of a workspace the
library allocates.

Checked through the C ABI against rf_decode_attention (which allocates its
workspace) on two calls in a row, within the attention tolerance the other GPU
tests use: max|o - o_ref| <= 1e-4 * max|o_ref| + 1e-6.  This file sorts last so a
run that stops at the first failure has already run every other test; it does
not depend on them and passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from ramforge_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(fn, q, k, v, ctx, H, KV, hd, batch, out):
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx, H, KV, hd, batch, out.data_ptr(), None)
    return rc


# (4096, 64, 32, 8, 128): 64 sequences x 8 KV heads need 266,240 floats per split,
# so the fixed scratch holds 15 splits, not the 64 rf_decode_attention uses: the
# reduced-split path (different chunking and merge order, same tolerance).
@pytest.mark.parametrize("ctx,batch,H,KV,hd", [(2048, 1, 32, 8, 128), (513, 8, 32, 8, 128), (32768, 1, 32, 8, 128),
                                               (300, 2, 32, 4, 64), (7, 3, 4, 2, 2), (4096, 64, 32, 8, 128)])
def test_noalloc_matches_allocating_entry_point_twice(ctx, batch, H, KV, hd):
    import torch
    L = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(ctx * 31 + batch)
    q = torch.randn(batch, H, hd, device="cuda", generator=g)
    k = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    v = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    ref = torch.empty(batch, H, hd, device="cuda")
    _lib.check(_call(L.rf_decode_attention, q, k, v, ctx, H, KV, hd, batch, ref))
    outs = []
    for _ in range(2):  # the scratch keeps the previous call's contents
        o = torch.full((batch, H, hd), float("nan"), device="cuda")
        _lib.check(_call(L.rf_decode_attention_noalloc, q, k, v, ctx, H, KV, hd, batch, o))
        outs.append(o)
    torch.cuda.synchronize()
    r = ref.cpu().numpy()
    tol = 1e-4 * np.abs(r).max() + 1e-6
    for o in outs:
        assert np.abs(o.cpu().numpy() - r).max() <= tol


def test_noalloc_rejects_shapes_beyond_its_scratch():
    import torch
    L = _lib.lib()
    batch, H, KV, hd, ctx = 64, 64, 64, 128, 32768  # 64 seqs x 64 heads x 64 splits x 130 floats > 16 MiB
    q = torch.zeros(1, device="cuda")
    out = torch.zeros(1, device="cuda")
    rc = L.rf_decode_attention_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), ctx, H, KV, hd, batch,
                                       out.data_ptr(), None)
    assert rc == _lib.RF_EINVAL
    assert b"fixed scratch" in L.rf_last_error()
