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

import ctypes as _ctypes

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


def _check_reshape(V: torch.Tensor, axis: int, block_size: int) -> None:
    """The reference blocks V with reshape(*rest, -1, block_size) (mxq/block/_driver.py:23-32), which torch refuses
    for an empty V whose other dimensions include a zero; the same RuntimeError here."""
    if V.numel() == 0:
        rest = [s for i, s in enumerate(V.shape) if i != axis]
        if 0 in rest:
            raise RuntimeError(f"cannot reshape tensor of 0 elements into shape {rest + [-1, block_size]} because the "
                               "unspecified dimension size -1 can be any value and is ambiguous")


def _blocked_shape(V, axis, nb, last):
    return tuple(V.shape[:axis]) + tuple(V.shape[axis + 1:]) + (nb, last)


def to_blocks(V: torch.Tensor, axis: int, block_size: int, X: Optional[torch.Tensor] = None) -> Blocks:
    """V moved to (..., nblocks, block_size), zero-padded; divided by the blocked scales X when given."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    _check_reshape(V, axis_, block_size)
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
    _check_reshape(V, axis_, block_size)
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


STREAM_MIN_BYTES = 8 << 20        # host tensors at least this large are streamed through the device in chunks
STREAM_CHUNK_BYTES = 16 << 20     # V bytes per chunk
STREAM_DEPTH = 3                  # chunks in flight: one copying in, one quantizing, one copying out
_streams = {}


def _copy_streams(dev):
    if dev not in _streams:
        _streams[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _streams[dev]


def _runs(total: int, per: int):
    """[start, stop) runs of at most `per` units covering range(total), their sizes ramping up from per / 8 at the start
    and back down at the end: the first copy in and the last copy out, which nothing overlaps, stay short."""
    head = [max(1, per >> 3), max(1, per >> 2), max(1, per >> 1)]
    if total <= 2 * sum(head) + per:
        sizes = [per] * (total // per) + ([total % per] if total % per else [])
    else:
        middle = total - 2 * sum(head)
        sizes = head + [per] * (middle // per) + ([middle % per] if middle % per else []) + head[::-1]
    runs, at = [], 0
    for n in sizes:
        runs.append((at, at + n))
        at += n
    return runs


def _quantize_streamed(V, spec, axis_, outer, L, inner, nb, block_size, dev):
    """A host V quantized through the device in independent chunks, copies in, kernels and copies out on three
    streams so PCIe carries both directions while the device quantizes. Chunks are whole outer slices when
    outer > 1, else runs of whole blocks along the axis; either way each chunk's V, P and X are contiguous ranges
    of the host tensors. Returns pinned host P and X after the last copy has landed."""
    import ctypes
    src = V.contiguous()
    if src.dtype != torch.float32:
        src = src.to(torch.float32)
    xshape = list(V.shape)
    xshape[axis_] = nb
    P = torch.empty(V.shape, dtype=torch.float32, pin_memory=True)
    X = torch.empty(xshape, dtype=torch.float32, pin_memory=True)
    vf, pf, xf = src.reshape(-1), P.reshape(-1), X.reshape(-1)
    chunks = []                        # (v0, v1, x0, x1, (outer, len, inner)) per chunk
    if outer > 1 and 4 * L * inner <= STREAM_CHUNK_BYTES:       # whole outer slices
        per = max(1, STREAM_CHUNK_BYTES // (4 * L * inner))
        for o0, o1 in _runs(outer, per):
            chunks.append((o0 * L * inner, o1 * L * inner, o0 * nb * inner, o1 * nb * inner, (o1 - o0, L, inner)))
    else:                              # runs of whole blocks inside each outer slice (the last may be short)
        per = max(1, STREAM_CHUNK_BYTES // (4 * block_size * inner))
        for o in range(outer):
            for b0, b1 in (_runs(nb, per) if outer == 1 else [(b, min(nb, b + per)) for b in range(0, nb, per)]):
                r0, r1 = b0 * block_size, min(L, b1 * block_size)
                vb, xb = o * L * inner, o * nb * inner
                chunks.append((vb + r0 * inner, vb + r1 * inner, xb + b0 * inner, xb + b1 * inner, (1, r1 - r0, inner)))
    cap_v = max(c[1] - c[0] for c in chunks)
    cap_x = max(c[3] - c[2] for c in chunks)
    h2d, comp, d2h = _copy_streams(dev)
    cur = torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        for s in (h2d, comp, d2h):
            s.wait_stream(cur)
        with torch.cuda.stream(comp):
            dv = [torch.empty(cap_v, dtype=torch.float32, device=dev) for _ in range(STREAM_DEPTH)]
            dp = [torch.empty(cap_v, dtype=torch.float32, device=dev) for _ in range(STREAM_DEPTH)]
            dx = [torch.empty(cap_x, dtype=torch.float32, device=dev) for _ in range(STREAM_DEPTH)]
        free = [None] * STREAM_DEPTH
        for i, (v0, v1, x0, x1, shape) in enumerate(chunks):
            s = i % STREAM_DEPTH
            nv = v1 - v0
            with torch.cuda.stream(h2d):
                if free[s] is not None:
                    h2d.wait_event(free[s])
                dv[s][:nv].copy_(vf[v0:v1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(landed)
                _lib.call("mxq_block_quantize", _lib.ptr(dv[s]), _lib.ptr(dp[s]), _lib.ptr(dx[s]), *shape,
                          block_size, ctypes.byref(spec), ctypes.c_void_p(comp.cuda_stream))
                done = torch.cuda.Event()
                done.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                pf[v0:v1].copy_(dp[s][:nv], non_blocking=True)
                xf[x0:x1].copy_(dx[s][:x1 - x0], non_blocking=True)
                free[s] = torch.cuda.Event()
                free[s].record(d2h)
        d2h.synchronize()
    _lib.check_waits()
    return P, X


def quantize_fused(V: torch.Tensor, spec: "_lib.MxqQuantSpec", axis: int, block_size: int):
    """A named quantizer's compose as one kernel: P and X from V in one pass (mxq_block_quantize). A large host V
    streams through the device in chunks (_quantize_streamed) and P, X come back as pinned host tensors."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    _check_reshape(V, axis_, block_size)
    home = _lib.home(V)
    dev = _lib.device_for(V)
    if _lib._wait_word is None:                             # the kernel's wait-status word, checked by every call
        _lib.wait_word()
    if not V.is_cuda and V.numel() * 4 >= STREAM_MIN_BYTES:
        return _quantize_streamed(V, spec, axis_, outer, L, inner, nb, block_size, dev)
    v = _lib.on(V, dev)
    P = torch.empty_like(v)
    xshape = list(V.shape)
    xshape[axis_] = nb
    X = torch.empty(xshape, dtype=torch.float32, device=dev)
    _lib.run("mxq_block_quantize", dev, _lib.ptr(v), _lib.ptr(P), _lib.ptr(X), outer, L, inner, block_size,
             _ctypes.byref(spec))
    if home == dev:
        return P, X
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


# ---------------------------------------------------------------------------------------- compact form
def _packed_shape(shape, e: int, m: int):
    """The codes tensor of the compact form: P's shape, the innermost extent halved for FP4 (two codes a byte)."""
    shape = list(shape)
    if e + m == 3:
        if not shape or shape[-1] % 2:
            raise ValueError(f"compact FP4 codes pair up along the innermost dimension, which is {shape[-1:]}")
        shape[-1] //= 2
    return shape


def quantize_packed(V: torch.Tensor, spec: "_lib.MxqQuantSpec", axis: int, block_size: int):
    """A named quantizer's codes and scales in the compact form (no reference counterpart): codes as the element
    format's OCP bit patterns (uint8; FP4 two per byte, the even element low) in P's layout, scales as E8M0 bytes
    (2^(b - 127), 0xFF NaN) in X's layout. ValueError when a code or a scale has no such byte."""
    import ctypes
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    _check_reshape(V, axis_, block_size)
    home = _lib.home(V)
    dev = _lib.device_for(V)
    v = _lib.on(V, dev)
    codes = torch.empty(_packed_shape(V.shape, spec.e, spec.m), dtype=torch.uint8, device=dev)
    xshape = list(V.shape)
    xshape[axis_] = nb
    scales = torch.empty(xshape, dtype=torch.uint8, device=dev)
    st = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.run("mxq_block_quantize_packed", dev, _lib.ptr(v), _lib.ptr(codes), _lib.ptr(scales), outer, L, inner,
             block_size, ctypes.byref(spec), _lib.ptr(st))
    bits = int(st.item())
    if bits & 4:
        raise RuntimeError("compact form: a tile's load did not arrive within the kernel's bounded wait; the codes "
                           "are undefined")
    if bits & 1:
        raise ValueError("compact form: a code is Inf or NaN, which this element format cannot hold")
    if bits & 2:
        raise ValueError("compact form: a scale is not a power of two an E8M0 byte can hold (an all-zero block "
                         "under the scale floor?)")
    return _lib.back(codes, home), _lib.back(scales, home)


def unpack(codes: torch.Tensor, scales: torch.Tensor, fmt) -> Tuple[torch.Tensor, torch.Tensor]:
    """(P, X) float32 from the compact form, codes in P's layout (FP4: two per byte) and scales in X's."""
    from ..element_quant.formats import get
    f = get(fmt)
    if f is None or codes.dtype != torch.uint8 or scales.dtype != torch.uint8:
        raise ValueError("unpack: uint8 codes and scales of an MX element format")
    home = _lib.home(codes)
    dev = _lib.device_for(codes, scales)
    c, x = codes.to(dev).contiguous(), scales.to(dev).contiguous()
    shape = list(c.shape)
    if f.e + f.m == 3:
        shape[-1] *= 2
    P = torch.empty(shape, dtype=torch.float32, device=dev)
    X = torch.empty(x.shape, dtype=torch.float32, device=dev)
    _lib.run("mxq_unpack", dev, _lib.ptr(c), _lib.ptr(x), _lib.ptr(P), _lib.ptr(X), P.numel(), X.numel(), f.e, f.m)
    return _lib.back(P, home), _lib.back(X, home)


def dequantize_packed(codes: torch.Tensor, scales: torch.Tensor, fmt, axis: int = 0,
                      block_size: int = BLOCK) -> torch.Tensor:
    """dequantize straight from the compact form: each code's value times its block's scale, float32."""
    from ..element_quant.formats import get
    f = get(fmt)
    if f is None or codes.dtype != torch.uint8 or scales.dtype != torch.uint8:
        raise ValueError("dequantize_packed: uint8 codes and scales of an MX element format")
    shape = list(codes.shape)
    if f.e + f.m == 3:
        shape[-1] *= 2
    ref = torch.empty(shape, dtype=torch.float32, device="meta")
    axis_, outer, L, inner, nb = _layout(ref, axis, block_size)
    home = _lib.home(codes)
    dev = _lib.device_for(codes, scales)
    c, x = codes.to(dev).contiguous(), scales.to(dev).contiguous()
    if x.numel() != outer * nb * inner:
        raise ValueError(f"dequantize_packed: scales of shape {tuple(scales.shape)} do not match codes {tuple(shape)}")
    out = torch.empty(shape, dtype=torch.float32, device=dev)
    _lib.run("mxq_dequantize_packed", dev, _lib.ptr(c), _lib.ptr(x), _lib.ptr(out), outer, L, inner, block_size, f.e,
             f.m)
    return _lib.back(out, home)
