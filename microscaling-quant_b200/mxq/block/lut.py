"""mxq.block.lut — MX-Gemmini's LUT operand (mxq/block/lut.py:23-34): block.mxgemmini, then each code replaced by
its column group's nearest table entry, one 16-entry table per 2^group columns of the K×n operand. Every setting is
keyword-required, as in the reference.

    P, X = quantize(V, "MXFP6_E3M2", axis=0, block_size=32, rounding_mode="rne", scale_floor=2**-23,
                    group=1, max_iters=50)                                V_hat = P * expand(X)

Three kernels: the fused block quantizer, the table fit, and pick with lookup fused; an axis-1 operand is read
transposed in place, never copied.
"""
import torch

from . import _driver, mxgemmini
from .. import lut

__all__ = ["quantize", "dequantize"]


def quantize(V: torch.Tensor, fmt, axis: int, block_size: int, *, rounding_mode: str, scale_floor: float,
             group: int, max_iters: int):
    """block.mxgemmini.quantize, then each code replaced by its table entry. Returns (P, X), float32."""
    if V.ndim != 2 or axis not in (0, 1, -1, -2):
        raise ValueError(f"block.lut: V must be 2-D with axis 0 or 1, got shape {tuple(V.shape)}, axis {axis}")
    lut.formats._format(fmt)                                   # refuse a non-LUT format first
    P, X = mxgemmini.quantize(V, fmt, axis=axis, block_size=block_size, rounding_mode=rounding_mode,
                              scale_floor=scale_floor)
    Pk = P if axis % 2 == 0 else P.t()                         # K×n (a view for axis 1)
    T = lut.tables(Pk, fmt, group=group, max_iters=max_iters)
    P_lut = lut.kmeans.pick_lookup(Pk, T, group=group)
    return (P_lut if axis % 2 == 0 else P_lut.t()).contiguous(), X


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = _driver.BLOCK) -> torch.Tensor:
    """V_hat = P * expand(X): each scale repeated block_size times along `axis`, cut to P's length."""
    return _driver.dequantize(P, X, axis, block_size)
