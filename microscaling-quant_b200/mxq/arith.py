"""Arithmetic helpers of a PE between quantizations (mxq/arith.py:68-137), each one libmxq_b200 kernel:

    exact_add(a, b, e, m)         a + b exactly, then one rounding to float(e, m); a zero addend returns the other
    truncate_significand(x, m)    keep m fraction bits of |x|'s significand (subnormals normalised first)
    flush_product(x, floor_exp)   |x| < 2^floor_exp -> +0
    saturate(x, limit, value)     |x| > limit -> sign(x) * value; -0 -> +0
"""
import numpy as np
import torch

from . import _lib
from .element_quant.float_em import GRIDS

__all__ = ["exact_add", "truncate_significand", "flush_product", "saturate"]


def _unary(name, x, *args):
    home = _lib.home(x)
    dev = _lib.device_for(x)
    t = _lib.on(x, dev)
    out = torch.empty_like(t)
    _lib.run(name, dev, _lib.ptr(t), _lib.ptr(out), t.numel(), *args)
    return _lib.back(out, home)


def exact_add(a: torch.Tensor, b: torch.Tensor, e: int, m: int, rounding_mode: str = "rne",
              grid: str = "ieee") -> torch.Tensor:
    from .rounding import mode_code
    code = mode_code(rounding_mode, "rounding_mode")
    if grid not in GRIDS:
        raise ValueError(f"grid must be one of {GRIDS}, got {grid!r}")
    for t in (a, b):
        if isinstance(t, torch.Tensor) and t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise TypeError(f"mxq_b200 exact_add takes float32 operands (values on a float grid), got {t.dtype}")
    home = _lib.home(a, b)
    dev = _lib.device_for(a, b)
    x, y = (t.contiguous() for t in torch.broadcast_tensors(_lib.on(a, dev), _lib.on(b, dev)))
    out = torch.empty_like(x)
    _lib.run("mxq_exact_add", dev, _lib.ptr(x), _lib.ptr(y), _lib.ptr(out), x.numel(), e, m, code, GRIDS.index(grid))
    return _lib.back(out, home)


def truncate_significand(x: torch.Tensor, m: int) -> torch.Tensor:
    return _unary("mxq_truncate_significand", x, int(m))


def flush_product(x: torch.Tensor, floor_exp: int) -> torch.Tensor:
    return _unary("mxq_flush_product", x, float(np.float32(2.0 ** floor_exp)))


def saturate(x: torch.Tensor, limit: float, value: float) -> torch.Tensor:
    return _unary("mxq_saturate", x, float(np.float32(limit)), float(np.float32(value)))
