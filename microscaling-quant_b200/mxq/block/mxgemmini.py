"""mxq.block.mxgemmini — MX-Gemmini's operand codes (mxq/block/mxgemmini.py:37-59): scale_factor.mxquant with
`scale_floor`, then the OCP element grid with `rounding_mode` (default ties away), optionally pre-rounded on the
ieee grid to `via`=(e, m). One fused kernel.

    P, X = quantize(V, "MXFP8_E4M3", axis=0)        V_hat = P * expand(X)
"""
from typing import Optional, Tuple, Union

import numpy as np
import torch

from .. import _lib, scale_factor
from . import _driver
from ..element_quant.formats import Format, get
from ..rounding import mode_code

__all__ = ["quantize", "dequantize"]


def spec(fmt, rounding_mode="ties_away", scale_floor=scale_factor.MXQUANT_FLOOR, via=None) -> "_lib.MxqQuantSpec":
    f = get(fmt)
    if f is None:
        return _lib.MxqQuantSpec(0, 0, 0, 0, 0.0, 0, 0.0, 0, 0)
    code = mode_code(rounding_mode, "rounding_mode")
    ve, vm = (0, 0) if via is None else (int(via[0]), int(via[1]))
    if via is not None and (ve, vm) != (8, 23) and not (1 <= ve <= 8 and 1 <= vm <= 22):
        raise ValueError(f"unsupported widths e={ve}, m={vm}")
    return _lib.MxqQuantSpec(2, f.e, f.m, code, float(np.float32(scale_floor)), 0, 0.0, ve, vm)


_spec = _lib.cached(spec)                  # quantize's own calls share one struct per argument set

def quantize(V: torch.Tensor, fmt: Union[str, Format], axis: int = 0, block_size: int = _driver.BLOCK,
             rounding_mode: str = "ties_away",
             scale_floor: float = scale_factor.MXQUANT_FLOOR,
             via: Optional[Tuple[int, int]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """MX-Gemmini block quantize V along `axis`. Returns (P codes, X power-of-two scales), float32."""
    return _driver.quantize_fused(V, _spec(fmt, rounding_mode, scale_floor, via), axis, block_size)


def quantize_packed(V: torch.Tensor, fmt: Union[str, Format], axis: int = 0, block_size: int = _driver.BLOCK,
                    rounding_mode: str = "ties_away",
                    scale_floor: float = scale_factor.MXQUANT_FLOOR) -> Tuple[torch.Tensor, torch.Tensor]:
    """quantize's codes and scales in the compact form (no reference counterpart): uint8 OCP bit patterns (FP4 two
    per byte) and E8M0 scale bytes; block.unpack gives back exactly quantize's (P, X). A block under the default
    scale floor (1e-38, not a power of two) has no E8M0 scale and raises ValueError; scale_floor=2**-127 or above,
    a power of two, always packs."""
    return _driver.quantize_packed(V, spec(fmt, rounding_mode, scale_floor), axis, block_size)


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = _driver.BLOCK) -> torch.Tensor:
    return _driver.dequantize(P, X, axis, block_size)
