"""The vector ops around the matmuls at a chosen precision (mxq/nn/_vector.py:48-89).

    None     as transformers computes them: softmax and RMSNorm in float32
    "bf16"   every step's result rounded to bf16 nearest-even right after the step (mxq.rounding.bf16, a kernel)

    op        steps rounded under "bf16"
    softmax   S - max, exp, sum, divide (S arrives scaled and masked)
    rmsnorm   x^2, mean, + eps, rsqrt, x * r, * weight

The steps and their order are transformers'; exp / rsqrt / the row sums are torch's float32 operations, the glue the
comparisons against the reference hold to a 1e-6 tolerance (their reduction order differs between devices).
EXACT is the Scheme with no quantization and float64 sums (FP32 pass-through codes, fp64_accum).
"""
from functools import partial
from typing import Callable, Optional

import torch

from .. import rounding
from .._fp64_accum import fp64_accum
from ..block import mxgemmini
from ..scheme import Scheme

__all__ = ["OPS", "PRECISIONS", "EXACT", "resolve", "rounder", "softmax", "rmsnorm"]

OPS = ("softmax", "rmsnorm")
PRECISIONS = (None, "bf16")

_PASSTHROUGH = partial(mxgemmini.quantize, fmt="FP32", axis=0)
EXACT = Scheme("exact", a=_PASSTHROUGH, b=_PASSTHROUGH, reduce=fp64_accum)


def resolve(vector) -> dict:
    """None | "bf16" (every op) | {op: None or "bf16"} -> {op: precision} for every op."""
    if vector is None or isinstance(vector, str):
        vector = {op: vector for op in OPS}
    if (not isinstance(vector, dict) or set(vector) - set(OPS)
            or any(not (v is None or (isinstance(v, str) and v in PRECISIONS)) for v in vector.values())):
        raise ValueError(f"vector must be None, 'bf16' or {{op: None or 'bf16'}} with op in {OPS}, got {vector!r}")
    return {op: vector.get(op) for op in OPS}


def rounder(precision: Optional[str]) -> Callable[[torch.Tensor], torch.Tensor]:
    """The rounding after each step, keeping the tensor's dtype: none (None) or bf16 nearest-even."""
    if precision is not None and not (isinstance(precision, str) and precision in PRECISIONS):
        raise ValueError(f"precision must be one of {PRECISIONS}, got {precision!r}")
    if precision is None:
        return lambda x: x
    return lambda x: rounding.bf16(x).to(x.dtype)


def softmax(S: torch.Tensor, precision: Optional[str]) -> torch.Tensor:
    """Softmax over the last dim of an already scaled and masked S."""
    if precision is None:
        return torch.softmax(S, dim=-1)
    r = rounder(precision)
    e = r(torch.exp(r(S - S.amax(dim=-1, keepdim=True))))
    return r(e / r(e.sum(dim=-1, keepdim=True)))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, precision: Optional[str]) -> torch.Tensor:
    """transformers' RMSNorm forward with a rounding after each step (None: none)."""
    r = rounder(precision)
    dtype = x.dtype
    h = x.to(torch.float32)
    v = r(r(h.pow(2)).mean(-1, keepdim=True))
    h = r(h * r(torch.rsqrt(r(v + eps))))
    return r(weight * h.to(dtype))
