"""A TMA wait that gives up is an error, not silent output: the test-only entry point runs the quantizer kernel
with its loads never issued and a short wait bound (nothing is in flight when the CTAs leave), and checks that
every lost tile is written as NaN, that the wait-status word and the device counter count the tiles, that the next
library call raises RuntimeError, and that the library works again once the word is cleared."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _device_timeouts():
    from mxq import _lib
    n = ctypes.c_uint32(0)
    _lib.call("mxq_device_timeouts", ctypes.byref(n))
    return n.value


def test_lost_tiles_raise():
    from mxq import _lib, block
    dev = torch.device("cuda", 0)
    V = torch.randn(64, 512, device=dev)
    word = _lib.wait_word()
    assert word.value == 0
    before = _device_timeouts()
    P = torch.zeros_like(V)
    X = torch.zeros(64, 16, device=dev)
    _lib.call("mxq_testing_wait_timeout", _lib.ptr(V), _lib.ptr(P), _lib.ptr(X), 64, 512, 64, _lib.stream(dev))
    torch.cuda.synchronize()
    tiles = (64 // 32) * (512 // 256)
    try:
        assert word.value == tiles
        assert _device_timeouts() - before == tiles
        assert torch.isnan(P).all() and torch.isnan(X).all()
        with pytest.raises(RuntimeError, match="gave up"):
            block.mxgemmini.quantize(V, "MXFP8_E4M3", axis=1)
    finally:
        _lib.clear_waits()
    P2, X2 = block.mxgemmini.quantize(V, "MXFP8_E4M3", axis=1)
    torch.cuda.synchronize()
    assert not torch.isnan(P2).any() and not torch.isnan(X2).any()
    assert word.value == 0
