"""mxq.block.ocp — OCP Microscaling v1.0 block quantization (mxq/block/ocp.py:35-49): the shared exponent
floor(log2 amax) - emax with E8M0 range handling, then the microxcaling element step (saturate, subnormals kept).
`rounding_mode` uses microxcaling's names ("even" RNE, "nearest" ties away, "floor"); `placement` picks the scale
rule (top | below_top | no_clip). One fused kernel.

    P, X = quantize(V, "MXFP8_E4M3", axis=0)        V_hat = P * expand(X)
"""
from typing import Tuple, Union

import torch

from .. import _lib, scale_factor
from . import _driver
from ..element_quant.formats import Format, get
from ..element_quant.microsoft import round_code

__all__ = ["quantize", "dequantize", "PLACEMENTS"]

PLACEMENTS = ("top", "below_top", "no_clip")


def spec(fmt, rounding_mode="even", scale_bits=8, placement="top") -> "_lib.MxqQuantSpec":
    f = get(fmt)
    if placement not in PLACEMENTS:
        raise ValueError(f"placement must be one of {PLACEMENTS}, got {placement!r}")
    if f is None:
        return _lib.MxqQuantSpec(0, 0, 0, 0, 0.0, 0, 0.0, 0, 0)
    return _lib.MxqQuantSpec(3, f.e, f.m, round_code(rounding_mode), 0.0, PLACEMENTS.index(placement),
                             scale_factor.scale_emax(scale_bits), 0, 0)


_spec = _lib.cached(spec)                  # quantize's own calls share one struct per argument set

def quantize(V: torch.Tensor, fmt: Union[str, Format], axis: int = 0, block_size: int = _driver.BLOCK,
             rounding_mode: str = "even", scale_bits: int = 8, placement: str = "top") -> Tuple[torch.Tensor, torch.Tensor]:
    """OCP block quantize V along `axis`. Returns (P codes, X power-of-two scales), float32."""
    return _driver.quantize_fused(V, _spec(fmt, rounding_mode, scale_bits, placement), axis, block_size)


def quantize_packed(V: torch.Tensor, fmt: Union[str, Format], axis: int = 0, block_size: int = _driver.BLOCK,
                    rounding_mode: str = "even", scale_bits: int = 8,
                    placement: str = "top") -> Tuple[torch.Tensor, torch.Tensor]:
    """quantize's codes and scales in the compact form (no reference counterpart): uint8 OCP bit patterns (FP4 two
    per byte) and E8M0 scale bytes; block.unpack gives back exactly quantize's (P, X)."""
    return _driver.quantize_packed(V, spec(fmt, rounding_mode, scale_bits, placement), axis, block_size)


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = _driver.BLOCK) -> torch.Tensor:
    return _driver.dequantize(P, X, axis, block_size)
