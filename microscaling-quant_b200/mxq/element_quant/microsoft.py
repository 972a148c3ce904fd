"""The microxcaling element step (mxq/element_quant/microsoft.py:18-23, restating microxcaling
_quantize_elemwise_core with saturate_normals=True, allow_denorm=True): per-element floor(log2|z|) clipped at the
format's min exponent, round ("nearest" ties away, "even" RNE, "floor" toward zero), saturate at max_norm.
The element step of block.ocp. FP32 (pass-through) has no element format and is rejected.
"""
from typing import Union

import torch

from .. import _lib
from .formats import Format, get

__all__ = ["quantize"]

ROUNDS = ("nearest", "floor", "even")


def round_code(rounding_mode: str) -> int:
    if rounding_mode == "dither":
        raise ValueError("mxq_b200: round method 'dither' draws random numbers and has no bit-exact kernel")
    if rounding_mode not in ROUNDS:
        raise ValueError(f"Unrecognized round method {rounding_mode}")
    return ROUNDS.index(rounding_mode)


def quantize_core(z: torch.Tensor, bits: int, exp_bits: int, max_norm: float, rounding_mode: str,
                  saturate_normals: bool) -> torch.Tensor:
    """_quantize_elemwise_core with allow_denorm=True, any (bits, exp_bits, max_norm)."""
    code = round_code(rounding_mode)
    home = _lib.home(z)
    dev = _lib.device_for(z)
    x = _lib.on(z, dev)
    out = torch.empty_like(x)
    _lib.run("mxq_microsoft", dev, _lib.ptr(x), _lib.ptr(out), x.numel(), bits, exp_bits, float(max_norm), code,
             int(bool(saturate_normals)))
    return _lib.back(out, home)


def quantize(z: torch.Tensor, fmt: Union[str, Format], rounding_mode: str = "even") -> torch.Tensor:
    f = get(fmt)
    if f is None:
        raise ValueError(f"{fmt!r} is pass-through (no element format); nothing to quantize")
    return quantize_core(z, f.m + 2, f.e, f.max_norm, rounding_mode, True)
