"""mxq.block.lut — MX-Gemmini's LUT operand (placeholder until the LUT kernels land)."""
from . import _driver

__all__ = ["quantize", "dequantize"]


def quantize(*args, **kwargs):
    raise NotImplementedError("mxq_b200: block.lut is not built yet")


def dequantize(P, X, axis: int = 0, block_size: int = _driver.BLOCK):
    return _driver.dequantize(P, X, axis, block_size)
