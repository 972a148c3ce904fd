"""What a LUT may hold and how the chip's finder reads it (mxq/lut/formats.py:29-159), for the four MX-Gemmini LUT
element formats.

    decode(codes, fmt)               element codes -> float32 values
    values(fmt)                      the values a table may hold: finite, and distinct to the finder
    encode(T, fmt)                   exact values -> element codes (the lowest code of each); raises on a missing one
    finder(codes, T, fmt, group=G)   the chip's index for each code: nearest in fixed point, |difference| masked,
                                     ties to the lower index

The format tables are built once per format by the library (mxq_lut_format_tables); decode, encode and finder are
CUDA kernels.
"""
import ctypes
from functools import lru_cache
from typing import Union

import numpy as np
import torch

from .. import _lib
from ..element_quant.formats import Format, get

__all__ = ["SIZE", "FORMATS", "decode", "values", "encode", "finder"]

SIZE = 16
FORMATS = ("MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "MXFP8_E4M3")


def _format(fmt: Union[str, Format]) -> Format:
    f = get(fmt)
    if f is None or f.name not in FORMATS:
        raise ValueError(f"mxq.lut: {fmt!r} is not a LUT format; MX-Gemmini sends {', '.join(FORMATS)} through LUTs")
    return f


@lru_cache(maxsize=None)
def _tables(name: str):
    """(every code's value float32, every code's fixed point int64, the finder-safe values float32 sorted)."""
    f = _format(name)
    n = 1 << (1 + f.e + f.m)
    vals = np.empty(n, np.float32)
    fx = np.empty(n, np.int64)
    safe = np.empty(256, np.float32)
    ns = ctypes.c_int32(0)
    _lib.call("mxq_lut_format_tables", f.e, f.m, vals.ctypes.data_as(ctypes.c_void_p), fx.ctypes.data_as(ctypes.c_void_p),
              safe.ctypes.data_as(ctypes.c_void_p), ctypes.byref(ns))
    return torch.from_numpy(vals), torch.from_numpy(fx), torch.from_numpy(safe[:ns.value].copy())


def _status(dev):
    return torch.zeros(1, dtype=torch.int32, device=dev)


def decode(codes: torch.Tensor, fmt: Union[str, Format]) -> torch.Tensor:
    """Element codes (integers) -> their float32 values."""
    f = _format(fmt)
    home = _lib.home(codes)
    dev = _lib.device_for(codes)
    c = _lib.on(codes, dev, torch.int64)
    out = torch.empty(c.shape, dtype=torch.float32, device=dev)
    st = _status(dev)
    _lib.run("mxq_lut_decode", dev, _lib.ptr(c), _lib.ptr(out), c.numel(), f.e, f.m, _lib.ptr(st))
    if int(st.item()):
        raise IndexError("mxq.lut.decode: a code is outside the format")
    return _lib.back(out, home)


def values(fmt: Union[str, Format]) -> torch.Tensor:
    """The values a table may hold, sorted ascending: finite, and no two with the same fixed point."""
    return _tables(_format(fmt).name)[2].clone()


def encode(T: torch.Tensor, fmt: Union[str, Format]) -> torch.Tensor:
    """Exact values -> element codes (the lowest code of each value). Raises on a value the format lacks."""
    f = _format(fmt)
    home = _lib.home(T)
    dev = _lib.device_for(T)
    v = _lib.on(T, dev)
    out = torch.empty(v.shape, dtype=torch.int64, device=dev)
    st = _status(dev)
    _lib.run("mxq_lut_encode", dev, _lib.ptr(v), _lib.ptr(out), v.numel(), f.e, f.m, _lib.ptr(st))
    if int(st.item()):
        bad = v.reshape(-1)[(out.reshape(-1) < 0).nonzero()[0, 0]].item()
        raise ValueError(f"mxq.lut: {bad!r} is not an exact {f.name} value, so it cannot be a table entry")
    return _lib.back(out, home)


def finder(codes: torch.Tensor, T: torch.Tensor, fmt: Union[str, Format], *, group: int) -> torch.Tensor:
    """The chip's index for each element code of a K×n tensor against its column group's table (T: (n >> group)
    × SIZE); nearest in the finder's fixed point, ties to the lower index. K×n int64."""
    f = _format(fmt)
    n = codes.shape[1]
    if T.shape[0] != n >> group or n % (1 << group):
        raise ValueError(f"mxq.lut.finder: {n} columns at group {group} need {n >> group} tables, got {T.shape[0]}")
    home = _lib.home(codes)
    dev = _lib.device_for(codes, T)
    c = _lib.on(codes, dev, torch.int64)
    t = _lib.on(T, dev)
    if t.shape[1] != SIZE:
        raise ValueError(f"mxq.lut.finder: tables must have {SIZE} entries, got {t.shape[1]}")
    out = torch.empty(c.shape, dtype=torch.int64, device=dev)
    st = _status(dev)
    _lib.run("mxq_lut_finder", dev, _lib.ptr(c), _lib.ptr(t), _lib.ptr(out), c.shape[0], n, group, f.e, f.m,
             _lib.ptr(st))
    s = int(st.item())
    if s & 1:                                            # the codes are indexed first (formats.py:152)
        raise IndexError("mxq.lut.finder: a code is outside the format")
    if s & 2:
        encode(t, f)                                     # raises with the offending value
    return _lib.back(out, home)
