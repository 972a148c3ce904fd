"""mxq.block.lut — MX-Gemmini's LUT operand (mxq/block/lut.py:23-34): block.mxgemmini, then each code replaced by
its column group's nearest table entry, one 16-entry table per 2^group columns of the K×n operand. Every setting is
keyword-required, as in the reference.

    P, X = quantize(V, "MXFP6_E3M2", axis=0, block_size=32, rounding_mode="rne", scale_floor=2**-23,
                    group=1, max_iters=50)                                V_hat = P * expand(X)

One C call (mxq_block_lut_quantize). Along axis 0 with blocks of 32 and whole 32-row blocks, one kernel quantizes V,
counts each code as it is made, fits each group's table, and writes every element's entry through the group's code ->
entry map; other row counts take the TMA quantizer writing the codes as bytes (their OCP bit patterns) and one kernel
that fits and looks up from the bytes; along axis 1 (the operand read transposed in place, never copied) and for other
block sizes the quantizer writes float codes, and the fit and a fused pick + lookup read them. Codes, tables and maps
live in a workspace.
"""
import ctypes

import torch

from . import _driver, mxgemmini
from .. import _lib, lut

__all__ = ["quantize", "dequantize"]


def quantize(V: torch.Tensor, fmt, axis: int, block_size: int, *, rounding_mode: str, scale_floor: float,
             group: int, max_iters: int):
    """block.mxgemmini.quantize, then each code replaced by its table entry. Returns (P, X), float32."""
    if V.ndim != 2 or axis not in (0, 1, -1, -2):
        raise ValueError(f"block.lut: V must be 2-D with axis 0 or 1, got shape {tuple(V.shape)}, axis {axis}")
    f = lut.formats._format(fmt)                               # refuse a non-LUT format first
    spec = mxgemmini.spec(fmt, rounding_mode, scale_floor)     # then what block.mxgemmini refuses
    _driver._layout(V, axis, block_size)
    _driver._check_reshape(V, axis % 2, block_size)
    lut.kmeans._check(V if axis % 2 == 0 else V.t(), group)    # then what lut.tables refuses
    if not isinstance(max_iters, int) or isinstance(max_iters, bool) or max_iters < 0:
        raise ValueError(f"mxq.lut: max_iters {max_iters!r} must be a non-negative integer")
    home = _lib.home(V)
    dev = _lib.device_for(V)
    v = _lib.on(V, dev)
    rows, cols = v.shape
    ax = axis % 2
    P = torch.empty_like(v)
    xshape = [rows, cols]
    xshape[ax] = (xshape[ax] + block_size - 1) // block_size
    X = torch.empty(xshape, dtype=torch.float32, device=dev)
    ws = torch.empty(max(1, _lib.lib().mxq_block_lut_workspace(rows, cols, ax, group)), dtype=torch.uint8,
                     device=dev)
    st = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.run("mxq_block_lut_quantize", dev, _lib.ptr(v), _lib.ptr(P), _lib.ptr(X), rows, cols, ax, block_size,
             ctypes.byref(spec), group, max_iters, _lib.ptr(ws), ws.numel(), _lib.ptr(st))
    bits = int(st.item())
    if bits & 4:
        raise RuntimeError("block.lut: a tile's load did not arrive within the quantizer's bounded wait")
    if bits:
        raise ValueError(f"mxq.lut: P holds a value that is not a {f.name} code; quantize it first")
    return _lib.back(P, home), _lib.back(X, home)


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = _driver.BLOCK) -> torch.Tensor:
    """V_hat = P * expand(X): each scale repeated block_size times along `axis`, cut to P's length."""
    return _driver.dequantize(P, X, axis, block_size)
