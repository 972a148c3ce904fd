"""mxq.rounding — the three rounding rules of the MX datapath (ties_away, rne, truncate), on float32 bit patterns
held in int64 (round_bits) or on integer-valued floats (round_int), and bf16 nearest-even on the bit pattern.

Same functions and semantics as the reference's mxq/rounding/__init__.py:51-85; each is one CUDA kernel of
libmxq_b200.so (mxq_round_bits, mxq_round_int_f32/f64, mxq_bf16).
"""
from typing import Union

import torch

from .. import _lib

MODES = ("ties_away", "rne", "truncate")
_CODE = {"ties_away": 0, "rne": 1, "truncate": 2}

__all__ = ["MODES", "round_bits", "round_int", "bf16", "ties_away", "rne", "truncate"]


def mode_code(mode: str, what: str = "mode") -> int:
    if mode not in _CODE:
        raise ValueError(f"{what} must be one of {MODES}, got {mode!r}")
    return _CODE[mode]


def round_bits(bits: torch.Tensor, keep: Union[int, torch.Tensor], mode: str) -> torch.Tensor:
    """A float32 bit pattern (int64 holding the uint32 pattern) rounded to `keep` fraction bits; `keep` an int or
    a tensor broadcast to `bits`, each in [0, 22]. Returns int64 patterns (mxq/rounding/__init__.py:51-55)."""
    code = mode_code(mode)
    home = _lib.home(bits)
    dev = _lib.device_for(bits, keep)
    b = _lib.on(bits, dev, torch.int64)
    if isinstance(keep, int) and not isinstance(keep, bool):
        if not 0 <= keep <= 22:
            raise ValueError("keep must be in [0, 22] (23 = identity is not a rounding)")
        k, ks = None, keep
    else:
        k = _lib.on(torch.as_tensor(keep), dev, torch.int64)
        b, k = (t.contiguous() for t in torch.broadcast_tensors(b, k))
        if bool((k < 0).any()) or bool((k > 22).any()):
            raise ValueError("keep must be in [0, 22] (23 = identity is not a rounding)")
        ks = 0
    out = torch.empty_like(b)
    _lib.run("mxq_round_bits", dev, _lib.ptr(b), _lib.ptr(k), ks, _lib.ptr(out), b.numel(), code)
    return _lib.back(out, home)


def _pattern(bits: torch.Tensor, drop, mask, half, mode: str) -> torch.Tensor:
    """One mode's bits(bits, drop, mask, half) (ties_away.py:5-6, rne.py:6-8, truncate.py:5-6): int64 patterns
    rounded with the caller's drop / mask / half (ints or int64 tensors broadcast against `bits`), the int64
    result not reduced to 32 bits. One kernel (mxq_round_pattern)."""
    code = mode_code(mode)
    home = _lib.home(bits)
    dev = _lib.device_for(bits, drop, mask, half)
    parts = [bits, drop, mask, half]
    shape = torch.broadcast_shapes(*(tuple(t.shape) for t in parts if isinstance(t, torch.Tensor)))
    args = []
    for i, t in enumerate(parts):
        if isinstance(t, torch.Tensor):
            args.append((_lib.on(t, dev, torch.int64).expand(shape).contiguous(), 0))
        elif i == 0:
            args.append((torch.full(shape, int(t), dtype=torch.int64, device=dev), 0))
        else:
            args.append((None, int(t)))
    out = torch.empty(shape, dtype=torch.int64, device=dev)
    (b, _), (d, ds), (m, ms), (h, hs) = args
    _lib.run("mxq_round_pattern", dev, _lib.ptr(b), _lib.ptr(d), ds, _lib.ptr(m), ms, _lib.ptr(h), hs, _lib.ptr(out),
             out.numel(), code)
    return _lib.back(out, home)


def round_int(k: torch.Tensor, mode: str) -> torch.Tensor:
    """An integer-valued float tensor rounded to an integer (mxq/rounding/__init__.py:58-61); float32 or float64."""
    code = mode_code(mode)
    home = _lib.home(k)
    if k.dtype not in (torch.float32, torch.float64):
        raise TypeError(f"mxq_b200 round_int computes in float32 or float64, got {k.dtype}")
    dev = _lib.device_for(k)
    x = _lib.on(k, dev, k.dtype)
    out = torch.empty_like(x)
    name = "mxq_round_int_f32" if x.dtype == torch.float32 else "mxq_round_int_f64"
    _lib.run(name, dev, _lib.ptr(x), _lib.ptr(out), x.numel(), code)
    return _lib.back(out, home)


def bf16(x: torch.Tensor) -> torch.Tensor:
    """float32 rounded to the bf16 grid, nearest-even, on the bit pattern; NaN passes through. Returns float32
    (mxq/rounding/__init__.py:64-85)."""
    home = _lib.home(x)
    dev = _lib.device_for(x)
    t = _lib.on(x, dev)
    out = torch.empty_like(t)
    _lib.run("mxq_bf16", dev, _lib.ptr(t), _lib.ptr(out), t.numel())
    return _lib.back(out, home)


from . import ties_away, rne, truncate  # noqa: E402  (the mode modules use _pattern and round_int above)
