"""pytest configuration: the `gpu` marker, import paths for the product package (microscaling-quant_b200/mxq)
and the test-only oracle (oracle/oracle.py)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "microscaling-quant_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(autouse=True)
def _no_lost_tiles(request):
    """After every GPU test: no bounded TMA wait gave up (a lost tile is written as NaN and would otherwise only show
    as wrong values). The timeout test clears what it provokes."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available() or not torch.cuda.is_initialized():
        return
    torch.cuda.synchronize()
    from mxq import _lib
    w = _lib._wait_word
    assert w is None or w.value == 0, f"{w.value} bounded TMA wait(s) gave up during this test"
