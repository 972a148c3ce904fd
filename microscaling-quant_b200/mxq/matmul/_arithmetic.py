"""The three rounding points inside a reducer, as one object (mxq/matmul/_arithmetic.py:41-211).

    product(a, b)          multiply two codes, round to the product format
    acc_add(S, p, e, m)    add product p into a running sum held in float(e, m)
    tile_add(C, tile)      add a finished, rescaled block sum into the output

    stage        MXQUANT(prod_e, prod_m)                         MXGEMMINI(prod_e=4, prod_m=3, prod_floor=-16)
    product      fp32 a*b, qtorch grid ties-away to the product  truncate to prod_m bits, flush below 2^prod_floor,
                 format                                          saturate with spike's (limit, value)
    acc_add      fp32 S+p, qtorch grid ties-away to the lane     S and p rounded RNE to the lane, exact sum, one RNE
    tile_add     fp32 C+tile                                     both rounded to bf16, exact sum rounded to bf16

An Arithmetic built by MXQUANT() or MXGEMMINI() carries `spec`, the machine-readable form the reducer kernels
read; its three callables run the same arithmetic as elementwise CUDA kernels. An Arithmetic built from other
callables has no kernel: the reducers refuse it rather than fall back to an unfused loop.
"""
from dataclasses import dataclass
from typing import Callable, Hashable, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _lib
from ..element_quant.float_em import bias

__all__ = ["Arithmetic", "MXQUANT", "MXGEMMINI", "compiled", "ArithSpec", "PROD_FLOOR"]

Tensor = torch.Tensor

#: products below 2^PROD_FLOOR flush to +0 (spike's mx_fp_math.h floor, for every product format)
PROD_FLOOR = -16


@dataclass(frozen=True)
class ArithSpec:
    """What the reducer kernels need to know about an Arithmetic (mirrors struct mxq_arith)."""
    kind: str                   # "mxquant" | "mxgemmini"
    prod_e: int
    prod_m: int
    prod_floor: Optional[int] = None
    sat_limit: float = 0.0
    sat_value: float = 0.0

    def c_struct(self) -> "_lib.MxqArith":
        """The struct the reducer entry points read (const): one per spec, built on first use."""
        return _c_struct(self)

    def _make_c_struct(self) -> "_lib.MxqArith":
        if self.kind == "mxquant":
            return _lib.MxqArith(0, self.prod_e, self.prod_m, 0, 0.0, 0.0, 0.0)
        thr = float(np.float32(2.0 ** self.prod_floor)) if self.prod_floor is not None else 0.0
        return _lib.MxqArith(1, self.prod_e, self.prod_m, int(self.prod_floor is not None), thr,
                             float(np.float32(self.sat_limit)), float(np.float32(self.sat_value)))


_c_struct = _lib.cached(ArithSpec._make_c_struct)


@dataclass(frozen=True)
class Arithmetic:
    name: str
    product: Callable[[Tensor, Tensor], Tensor]
    acc_add: Callable[[Tensor, Tensor, int, int], Tensor]
    tile_add: Callable[[Tensor, Tensor], Tensor]
    #: the reference's fusion hooks (systolic / anchor / adder use them when set); kept for API compatibility.
    #: The CUDA reducers are fused already, so `compiled` leaves them None.
    fused_reduction: Optional[Callable[[Sequence[Tuple[int, int]], int], Callable]] = None
    fused_block: Optional[Callable[[Sequence[Tuple[int, int]], int, int], Callable]] = None
    fuse: Optional[Callable[[Hashable, Callable], Callable]] = None
    #: the kernel form of this Arithmetic; None for one built from arbitrary callables
    spec: Optional[ArithSpec] = None


def _elementwise(name, spec, *tensors, extra=()):
    import ctypes
    home = _lib.home(*tensors)
    dev = _lib.device_for(*tensors)
    ts = [t.contiguous() for t in torch.broadcast_tensors(*[_lib.on(t, dev) for t in tensors])]
    out = torch.empty_like(ts[0])
    c = spec.c_struct()
    _lib.run(name, dev, *[_lib.ptr(t) for t in ts], _lib.ptr(out), out.numel(), ctypes.byref(c), *extra)
    return _lib.back(out, home)


def _from_spec(name: str, spec: ArithSpec) -> Arithmetic:
    return Arithmetic(
        name=name,
        product=lambda a, b: _elementwise("mxq_arith_product", spec, a, b),
        acc_add=lambda S, p, e, m: _elementwise("mxq_arith_acc_add", spec, S, p, extra=(int(e), int(m))),
        tile_add=lambda C, tile: _elementwise("mxq_arith_tile_add", spec, C, tile),
        spec=spec,
    )


def MXQUANT(prod_e: int, prod_m: int) -> Arithmetic:
    """MXQuant `_simulate_atw`: qtorch nearest of the fp32 product; fp32 add then qtorch nearest of the sum to the
    lane; fp32 cross-block add (mxq/matmul/_arithmetic.py:64-73)."""
    return _from_spec(f"mxquant(prod=e{prod_e}m{prod_m})", ArithSpec("mxquant", prod_e, prod_m))


def _saturation(prod_e: int, prod_m: int) -> Tuple[float, float]:
    """(limit, value) of spike's product saturation (mx_fp_math.h:42-56, as _arithmetic.py:88-102 states it): a
    product above max_normal becomes sign * sat_val. max_normal is 448 for e4m3, else 2^b (2 - 2^-m); sat_val is
    2^(b+1) (1 + (2^m - 2) / 2^m), Inf when that is beyond float32."""
    b = bias(prod_e)
    fp8 = (prod_e, prod_m) == (4, 3)
    top = 2 ** prod_m
    limit = 2.0 ** (b + 1 if fp8 else b) * (1 + ((top - 2) if fp8 else (top - 1)) / top)
    value = 2.0 ** (b + 1) * (1 + (top - 2) / top)
    if value > float(torch.finfo(torch.float32).max):
        value = float("inf")
    return limit, value


def MXGEMMINI(prod_e: int = 4, prod_m: int = 3, prod_floor: Optional[int] = PROD_FLOOR) -> Arithmetic:
    """MX-Gemmini's PE column as spike computes it (mxq/matmul/_arithmetic.py:111-134): product significand
    truncated to prod_m bits, flushed below 2^prod_floor (None: no flush), saturated; lanes rounded RNE (bf16 on the
    bits for (8, 7)) and added exactly; cross-block in bf16. Every lane rounding returns +0 for a zero."""
    limit, value = _saturation(prod_e, prod_m)
    return _from_spec(f"mxgemmini(prod=e{prod_e}m{prod_m})",
                      ArithSpec("mxgemmini", prod_e, prod_m, prod_floor, limit, value))


def compiled(arith: Arithmetic) -> Arithmetic:
    """The reference passes an Arithmetic through torch.compile to fuse its elementwise chains. The CUDA kernels
    are that fusion already (one kernel per reduction stage and one per whole reducer), so this returns the same
    arithmetic under the name compiled(...); results are unchanged."""
    return Arithmetic(name=f"compiled({arith.name})", product=arith.product, acc_add=arith.acc_add,
                      tile_add=arith.tile_add, spec=arith.spec)
