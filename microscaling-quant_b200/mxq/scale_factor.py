"""mxq.scale_factor — step 1 of block quantization: a power-of-two scale X = f(amax) per block
(mxq/scale_factor.py:40-81). Each rule is one libmxq_b200 kernel; amax is float32.

    mxquant(amax, floor)          2^floor(log2 max(amax, floor)), floored at `floor`
    ocp(amax, emax)               2^(floor(log2 amax) - emax), E8M0 range: NaN above, clamped below
    ocp_below_top(amax, emax)     ocp's scale times two
    ocp_no_clip(amax, fmt)        ocp's scale, doubled for the blocks whose max would clip

floor(log2 x) is taken as the reference computes it, floor of the correctly rounded float32 log2.
"""
import numpy as np
import torch

from . import _lib

__all__ = ["mxquant", "ocp", "ocp_below_top", "ocp_no_clip", "MXQUANT_FLOOR", "HARDWARE_FLOOR"]

#: MXQuant's simulation floor: a zero block gets a finite (float32 subnormal) scale
MXQUANT_FLOOR = 1e-38
#: MXQuant end_to_end_linear and the MX-Gemmini requantizer: FLT_EPSILON
HARDWARE_FLOOR = 2.0 ** -23


def _amax(amax):
    if amax.dtype != torch.float32:
        raise TypeError(f"mxq_b200 computes scale factors in float32, got {amax.dtype}")


def scale_emax(scale_bits: int) -> float:
    """float32(2^(scale_bits-1) - 1): the E8M0 exponent bound as torch compares it."""
    return float(np.float32(2 ** (scale_bits - 1) - 1))


def _run(name, amax, *args):
    _amax(amax)
    home = _lib.home(amax)
    dev = _lib.device_for(amax)
    a = _lib.on(amax, dev)
    out = torch.empty_like(a)
    _lib.run(name, dev, _lib.ptr(a), _lib.ptr(out), a.numel(), *args)
    return _lib.back(out, home)


def mxquant(amax: torch.Tensor, floor: float = MXQUANT_FLOOR) -> torch.Tensor:
    return _run("mxq_scale_mxquant", amax, float(np.float32(floor)))


def ocp(amax: torch.Tensor, emax: int, scale_bits: int = 8) -> torch.Tensor:
    return _run("mxq_scale_ocp", amax, int(emax), scale_emax(scale_bits))


def ocp_below_top(amax: torch.Tensor, emax: int, scale_bits: int = 8) -> torch.Tensor:
    return ocp(amax, emax - 1, scale_bits)


def ocp_no_clip(amax: torch.Tensor, fmt, rounding_mode: str = "even", scale_bits: int = 8) -> torch.Tensor:
    from .element_quant.formats import get
    from .element_quant.microsoft import round_code
    f = get(fmt)
    if f is None:
        raise ValueError(f"{fmt!r} is pass-through (no element format); it has no scale")
    return _run("mxq_scale_ocp_no_clip", amax, f.e, f.m, round_code(rounding_mode), scale_emax(scale_bits))
