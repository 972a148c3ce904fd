"""The product (the mxq package on CUDA) behind the oracle's function names, so one set of golden checks
(tests/test_oracle_golden.py) runs against both: the oracle on CPU, the CUDA kernels through the public API here.
Inputs are numpy arrays copied to cuda:0; results come back as numpy."""
import numpy as np
import torch

import mxq
from mxq import arith as _arith, block, matmul, rounding, scale_factor
from mxq.element_quant import float_em as _float_em, microsoft as _ms

DEV = "cuda"
FORMATS = {"MXFP8_E4M3": (4, 3, 8, 448.0), "MXFP8_E5M2": (5, 2, 15, 57344.0), "MXFP6_E3M2": (3, 2, 4, 28.0),
           "MXFP6_E2M3": (2, 3, 2, 7.5), "MXFP4": (2, 1, 2, 6.0)}
LUT_FORMATS = ("MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "MXFP8_E4M3")


def T(a, dtype=None):
    a = np.asarray(a)
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def N(t):
    return t.detach().cpu().numpy()


def round_bits(bits, keep, mode):
    k = int(keep) if np.isscalar(keep) else T(np.asarray(keep, np.int64))
    return N(rounding.round_bits(T(np.asarray(bits, np.int64)), k, mode))


def round_int(k, mode):
    return N(rounding.round_int(T(k), mode))


def bf16(x):
    return N(rounding.bf16(T(np.asarray(x, np.float32))))


def float_em(z, e, m, rounding_mode="ties_away", grid="qtorch"):
    return N(_float_em.quantize(T(z), e, m, rounding_mode, grid))


def microsoft(A, fmt, rounding_mode="even", saturate_normals=True):
    e, m, _, mn = FORMATS[fmt]
    return N(_ms.quantize_core(T(np.asarray(A, np.float32)), m + 2, e, mn, rounding_mode, saturate_normals))


def scale_mxquant(amax, floor=1e-38):
    return N(scale_factor.mxquant(T(np.asarray(amax, np.float32)), floor))


def scale_ocp(amax, emax, scale_bits=8):
    return N(scale_factor.ocp(T(np.asarray(amax, np.float32)), emax, scale_bits))


def scale_ocp_no_clip(amax, fmt, rounding_mode="even", scale_bits=8):
    return N(scale_factor.ocp_no_clip(T(np.asarray(amax, np.float32)), fmt, rounding_mode, scale_bits))


def exact_add(a, b, e, m, rounding_mode="rne", grid="ieee"):
    return N(_arith.exact_add(T(np.asarray(a, np.float32)), T(np.asarray(b, np.float32)), e, m, rounding_mode, grid))


def truncate_significand(x, m):
    return N(_arith.truncate_significand(T(np.asarray(x, np.float32)), m))


def flush_product(x, floor_exp):
    return N(_arith.flush_product(T(np.asarray(x, np.float32)), floor_exp))


def saturate(x, limit, value):
    return N(_arith.saturate(T(np.asarray(x, np.float32)), limit, value))


def block_quantize(V, family, fmt, axis=0, block_size=32, rounding_mode=None, scale_floor=1e-38, via=None,
                   scale_bits=8, placement="top"):
    Vt = T(np.asarray(V, np.float32))
    if fmt in (None, "FP32"):
        P, X = block.mxgemmini.quantize(Vt, "FP32", axis=axis, block_size=block_size)
    elif family == "mxquant":
        P, X = block.mxquant.quantize(Vt, fmt, axis=axis, block_size=block_size)
    elif family == "mxgemmini":
        P, X = block.mxgemmini.quantize(Vt, fmt, axis=axis, block_size=block_size,
                                        rounding_mode=rounding_mode or "ties_away", scale_floor=scale_floor, via=via)
    else:
        P, X = block.ocp.quantize(Vt, fmt, axis=axis, block_size=block_size, rounding_mode=rounding_mode or "even",
                                  scale_bits=scale_bits, placement=placement)
    return N(P), N(X)


def arith_mxgemmini(prod_e=4, prod_m=3, prod_floor=-16):
    return matmul.MXGEMMINI(prod_e, prod_m, prod_floor)


def arith_mxquant(prod_e, prod_m):
    return matmul.MXQUANT(prod_e, prod_m)


def _ops(P_A, X_A, P_B, X_B):
    return [T(np.asarray(t, np.float32)) for t in (P_A, X_A, P_B, X_B)]


def systolic(P_A, X_A, P_B, X_B, arith, schedule, size=16, block_size=32, threads=None):
    return N(matmul.systolic(*_ops(P_A, X_A, P_B, X_B), arith, schedule, size, block_size))


def adder_tree(P_A, X_A, P_B, X_B, arith, schedule, size=16, block_size=32, threads=None):
    return N(matmul.adder_tree(*_ops(P_A, X_A, P_B, X_B), arith, schedule, size, block_size))


def anchor_tree(P_A, X_A, P_B, X_B, arith, schedule=None, size=16, block_size=32, threads=None, **kw):
    return N(matmul.anchor_tree(*_ops(P_A, X_A, P_B, X_B), arith, schedule, size, block_size, **kw))


def fp64_accum(P_A, X_A, P_B, X_B, block_size=32, threads=None):
    return N(mxq.fp64_accum(*_ops(P_A, X_A, P_B, X_B), block_size))


# ------------------------------------------------------------------------------------------------------ LUT
from mxq import lut as _lut  # noqa: E402


def lut_format_tables(fmt):
    v, fx, s = _lut.formats._tables(fmt)
    return v.numpy(), fx.numpy(), s.numpy()


def lut_tables(P, fmt, group, max_iters):
    return N(_lut.tables(T(np.asarray(P, np.float32)), fmt, group=group, max_iters=max_iters))


def lut_pick(P, Tt, group):
    return N(_lut.pick(T(np.asarray(P, np.float32)), T(np.asarray(Tt, np.float32)), group=group))


def lut_lookup(I, Tt, group):
    return N(_lut.lookup(T(np.asarray(I, np.int64)), T(np.asarray(Tt, np.float32)), group=group))


def lut_encode(Tt, fmt):
    return N(_lut.encode(T(np.asarray(Tt, np.float32)), fmt))


def lut_decode(codes, fmt):
    return N(_lut.decode(T(np.asarray(codes, np.int64)), fmt))


def lut_finder(codes, Tt, fmt, group):
    return N(_lut.finder(T(np.asarray(codes, np.int64)), T(np.asarray(Tt, np.float32)), fmt, group=group))


def lut_block_quantize(V, fmt, axis, block_size, rounding_mode, scale_floor, group, max_iters):
    P, X = block.lut.quantize(T(np.asarray(V, np.float32)), fmt, axis, block_size, rounding_mode=rounding_mode,
                              scale_floor=scale_floor, group=group, max_iters=max_iters)
    return N(P), N(X)
