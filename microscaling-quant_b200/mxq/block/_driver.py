"""The block quantization driver (mxq/block/_driver.py:23-72): split a tensor into blocks along one axis, zero-pad,
run the two steps, put codes and scales back into the caller's layout.

    P, X = compose(V, scale=f, elem=g, axis=0, block_size=BLOCK)
    V_hat = dequantize(P, X, axis=0)

P has V's shape (the codes); X has V's shape with `axis` of length ceil(len / block_size) (the scales).

With caller-supplied steps, compose runs the reference's three stages as three kernels -- block max
(mxq_block_amax), the blocked and scaled values (mxq_to_blocks), the layout back (mxq_from_blocks) -- around the two
callables, which see the same (..., nblocks, block_size) tensors the reference hands them. The named quantizers
(block.mxquant / mxgemmini / ocp) skip all of that: `quantize_fused` is one kernel that reads V once and writes P
and X once (mxq_block_quantize).
"""
from typing import Callable, NamedTuple, Optional, Tuple

import torch

from .. import _lib

BLOCK = 32

__all__ = ["BLOCK", "compose", "dequantize", "Blocks", "to_blocks", "codes_from_blocks", "scales_from_blocks"]


class Blocks(NamedTuple):
    data: torch.Tensor   # (..., nblocks, block_size): the block axis moved last, zero-padded
    axis: int
    n: int               # original length along axis


def _layout(V: torch.Tensor, axis: int, block_size: int):
    """(axis, outer, len, inner, nblocks) of V viewed as [outer, len, inner] with blocks along len."""
    if not -V.ndim <= axis < V.ndim:
        raise IndexError(f"axis {axis} out of range for {V.ndim}-D tensor")
    if not isinstance(block_size, int) or block_size < 1:
        raise ValueError(f"block_size must be a positive integer, got {block_size!r}")
    axis = axis % V.ndim
    outer = 1
    for s in V.shape[:axis]:
        outer *= s
    inner = 1
    for s in V.shape[axis + 1:]:
        inner *= s
    L = V.shape[axis]
    return axis, outer, L, inner, (L + block_size - 1) // block_size


def _blocked_shape(V, axis, nb, last):
    return tuple(V.shape[:axis]) + tuple(V.shape[axis + 1:]) + (nb, last)


def to_blocks(V: torch.Tensor, axis: int, block_size: int, X: Optional[torch.Tensor] = None) -> Blocks:
    """V moved to (..., nblocks, block_size), zero-padded; divided by the blocked scales X when given."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    home = _lib.home(V)
    dev = _lib.device_for(V, X)
    v = _lib.on(V, dev)
    x = None if X is None else _lib.on(X, dev)
    Z = torch.empty(_blocked_shape(V, axis_, nb, block_size), dtype=torch.float32, device=dev)
    _lib.run("mxq_to_blocks", dev, _lib.ptr(v), _lib.ptr(x), _lib.ptr(Z), outer, L, inner, block_size)
    return Blocks(_lib.back(Z, home), axis_, L)


def codes_from_blocks(P: torch.Tensor, b: Blocks) -> torch.Tensor:
    """(..., nblocks, block_size) -> the original layout, padding removed."""
    nb, bs = P.shape[-2], P.shape[-1]
    lead = P.shape[:-2]
    shape = list(lead[:b.axis]) + [b.n] + list(lead[b.axis:])
    outer = 1
    for s in lead[:b.axis]:
        outer *= s
    inner = 1
    for s in lead[b.axis:]:
        inner *= s
    home = _lib.home(P)
    dev = _lib.device_for(P)
    src = _lib.on(P, dev)
    out = torch.empty(shape, dtype=torch.float32, device=dev)
    _lib.run("mxq_from_blocks", dev, _lib.ptr(src), _lib.ptr(out), outer, b.n, inner, bs)
    return _lib.back(out, home)


def scales_from_blocks(X: torch.Tensor, b: Blocks) -> torch.Tensor:
    """(..., nblocks, 1) -> V's layout with `axis` of length nblocks."""
    nb = X.shape[-2]
    return codes_from_blocks(X.reshape(*X.shape[:-2], 1, nb), Blocks(b.data, b.axis, nb))


def compose(V: torch.Tensor, *, scale: Optional[Callable[[torch.Tensor], torch.Tensor]],
            elem: Optional[Callable[[torch.Tensor], torch.Tensor]],
            axis: int = 0, block_size: int = BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    """Block quantization from its two steps (mxq/block/_driver.py:45-66). Returns (P codes, X scales), float32.

    scale(amax) -> X   amax is each block's max |value|, shape (..., nblocks, 1); X the same shape
    elem(z) -> P       z = block / X, shape (..., nblocks, block_size); P the same shape
    Either may be None: no scale step means X = 1, no element step means P = V / X."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    home = _lib.home(V)
    dev = _lib.device_for(V)
    v = _lib.on(V, dev)
    if scale is None:
        X = torch.ones(_blocked_shape(V, axis_, nb, 1), dtype=torch.float32, device=dev)
        Xb = None
    else:
        amax = torch.empty(_blocked_shape(V, axis_, nb, 1), dtype=torch.float32, device=dev)
        _lib.run("mxq_block_amax", dev, _lib.ptr(v), _lib.ptr(amax), outer, L, inner, block_size)
        X = scale(amax)
        Xb = X
    b = to_blocks(v, axis_, block_size, None if Xb is None else Xb.expand(amax.shape))
    z = b.data
    P = z.clone() if elem is None else elem(z)
    P_out = codes_from_blocks(P.to(torch.float32), b)
    X_out = scales_from_blocks(X.to(torch.float32).expand(_blocked_shape(V, axis_, nb, 1)), b)
    return _lib.back(P_out, home), _lib.back(X_out, home)


def quantize_fused(V: torch.Tensor, spec: "_lib.MxqQuantSpec", axis: int, block_size: int):
    """A named quantizer's compose as one kernel: P and X from V in one pass (mxq_block_quantize)."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    home = _lib.home(V)
    dev = _lib.device_for(V)
    v = _lib.on(V, dev)
    P = torch.empty_like(v)
    xshape = list(V.shape)
    xshape[axis_] = nb
    X = torch.empty(xshape, dtype=torch.float32, device=dev)
    import ctypes
    _lib.run("mxq_block_quantize", dev, _lib.ptr(v), _lib.ptr(P), _lib.ptr(X), outer, L, inner, block_size,
             ctypes.byref(spec))
    return _lib.back(P, home), _lib.back(X, home)


def dequantize(P: torch.Tensor, X: torch.Tensor, axis: int = 0, block_size: int = BLOCK) -> torch.Tensor:
    """V_hat = P * expand(X): each scale repeated block_size times along `axis`, cut to P's length."""
    axis_, outer, L, inner, nb = _layout(P, axis, block_size)
    home = _lib.home(P)
    dev = _lib.device_for(P, X)
    p = _lib.on(P, dev)
    x = _lib.on(X, dev)
    if x.numel() != outer * nb * inner:
        raise ValueError(f"dequantize: scales of shape {tuple(X.shape)} do not match codes {tuple(P.shape)}")
    out = torch.empty_like(p)
    _lib.run("mxq_dequantize", dev, _lib.ptr(p), _lib.ptr(x), _lib.ptr(out), outer, L, inner, block_size)
    return _lib.back(out, home)
