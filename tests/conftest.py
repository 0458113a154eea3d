"""Shared test setup.

Markers: `gpu` tests need a CUDA device (run with `-m gpu` on a B200); all
other tests run on CPU.  The oracle (oracle/) is the parity checker; the
product path is ramforge_b200 / librfcuda.so.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: large model / long-running case")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Compile the oracle and the native libraries once per session (no-op when fresh)."""
    from oracle import oracle as orc
    orc.build()
    from ramforge_b200 import build
    build.build_synth()
    build.build_cuda()


def _cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
