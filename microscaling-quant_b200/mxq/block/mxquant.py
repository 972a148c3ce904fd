"""mxq.block.mxquant — MXQuant's simulation codes (mxq/block/mxquant.py:26-32): scale_factor.mxquant (block max in
[1, 2)) then float_em on the qtorch 0.2.0 grid, ties away. One fused kernel.

    P, X = quantize(V, "MXFP8_E4M3", axis=0)        V_hat = P * expand(X)
"""
from typing import Tuple, Union

import numpy as np
import torch

from .. import _lib, scale_factor
from . import _driver
from ..element_quant.formats import Format, get

__all__ = ["quantize", "dequantize"]


def spec(fmt) -> "_lib.MxqQuantSpec":
    f = get(fmt)
    if f is None:
        return _lib.MxqQuantSpec(0, 0, 0, 0, 0.0, 0, 0.0, 0, 0)
    return _lib.MxqQuantSpec(1, f.e, f.m, 0, float(np.float32(scale_factor.MXQUANT_FLOOR)), 0, 0.0, 0, 0)


_spec = _lib.cached(spec)                  # quantize's own calls share one struct per argument set

def quantize(V: torch.Tensor, fmt: Union[str, Format], axis: int = 0,
             block_size: int = _driver.BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    """MXQuant-simulation block quantize V along `axis`. Returns (P codes, X power-of-two scales), float32."""
    return _driver.quantize_fused(V, _spec(fmt), axis, block_size)


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = _driver.BLOCK) -> torch.Tensor:
    return _driver.dequantize(P, X, axis, block_size)
