"""mxq.microxcaling — the OCP MX v1.0 element formats with Microsoft microxcaling's conversion semantics
(mxq/microxcaling/__init__.py and the vendored formats.py / elemwise.py / blockwise.py it wraps), computed by the
mxq_microsoft and block-quantizer kernels.

    fp8_e4m3(x)  fp8_e5m2(x)  fp6_e3m2(x)  fp6_e2m3(x)  fp4_e2m1(x)  bf16(x)    fake-quantized values
    quantize(x, fmt, round="even")                 any ElemFormat, MX conversion flags
    block_quantize(x, fmt, axis=-1, block_size=32, scale_bits=8, round="even")   _quantize_mx: P * 2^shared_exp
    params(fmt) -> (ebits, mbits, emax, max_norm, min_norm);  ElemFormat, RoundingMode
"""
from enum import Enum, IntEnum

from ..element_quant.microsoft import quantize_core as _core

__all__ = ["fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1", "bf16", "quantize", "block_quantize", "params",
           "ElemFormat", "RoundingMode"]

FP32_EXPONENT_BIAS = 127
FP32_MIN_NORMAL = 2 ** (-FP32_EXPONENT_BIAS + 1)


class RoundingMode(IntEnum):
    nearest = 0
    floor = 1
    even = 2

    @staticmethod
    def string_enums():
        return [s.name for s in list(RoundingMode)]


class ElemFormat(Enum):
    int8 = 1
    int4 = 2
    int2 = 3
    fp8_e5m2 = 4
    fp8_e4m3 = 5
    fp6_e3m2 = 6
    fp6_e2m3 = 7
    fp4 = 8
    fp4_e2m1 = 8
    float16 = 9
    fp16 = 9
    bfloat16 = 10
    bf16 = 10

    @staticmethod
    def from_str(s):
        assert s is not None, "String elem_format == None"
        s = s.lower()
        if hasattr(ElemFormat, s):
            return getattr(ElemFormat, s)
        raise Exception("Undefined elem format", s)


# (ebits, mbits incl. sign and implicit bit, emax) of each format (microxcaling formats.py:61-125)
_PARAMS = {ElemFormat.int8: (0, 8, 0), ElemFormat.int4: (0, 4, 0), ElemFormat.int2: (0, 2, 0),
           ElemFormat.fp8_e5m2: (5, 4, 15), ElemFormat.fp8_e4m3: (4, 5, 8), ElemFormat.fp6_e3m2: (3, 4, 4),
           ElemFormat.fp6_e2m3: (2, 5, 2), ElemFormat.fp4: (2, 3, 2), ElemFormat.float16: (5, 12, 15),
           ElemFormat.bfloat16: (8, 9, 127)}

#: formats with no Inf encoding: out-of-range values saturate to max_norm
_SATURATING = {ElemFormat.fp8_e4m3, ElemFormat.fp6_e3m2, ElemFormat.fp6_e2m3, ElemFormat.fp4_e2m1}


def params(fmt):
    """(ebits, mbits, emax, max_norm, min_norm) of an ElemFormat or its name."""
    if isinstance(fmt, str):
        fmt = ElemFormat.from_str(fmt)
    if fmt not in _PARAMS:
        raise Exception("Unknown element format %s" % fmt)
    ebits, mbits, emax = _PARAMS[fmt]
    max_norm = 2 ** emax * 1.75 if fmt == ElemFormat.fp8_e4m3 else 2 ** emax * float(2 ** (mbits - 1) - 1) / 2 ** (mbits - 2)
    min_norm = 0 if ebits == 0 else 2 ** (2 - 2 ** (ebits - 1))
    return ebits, mbits, emax, max_norm, min_norm


def _elemwise(x, fmt, round, saturate):
    ebits, mbits, _, max_norm, _ = params(fmt)
    return _core(x, mbits, ebits, max_norm, round, saturate)


def quantize(x, fmt, round="even"):
    """Quantize to any ElemFormat with OCP MX conversion semantics (saturate the formats without Inf)."""
    fmt = ElemFormat.from_str(fmt) if isinstance(fmt, str) else fmt
    return _elemwise(x, fmt, round, fmt in _SATURATING)


def fp8_e4m3(x, round="even"): return quantize(x, ElemFormat.fp8_e4m3, round)
def fp8_e5m2(x, round="even"): return quantize(x, ElemFormat.fp8_e5m2, round)
def fp6_e3m2(x, round="even"): return quantize(x, ElemFormat.fp6_e3m2, round)
def fp6_e2m3(x, round="even"): return quantize(x, ElemFormat.fp6_e2m3, round)
def fp4_e2m1(x, round="even"): return quantize(x, ElemFormat.fp4_e2m1, round)


def bf16(x, round="even"):
    """_quantize_bfloat(x, 16): 9 mantissa bits (sign and implicit included), 8 exponent bits, no saturation."""
    max_norm = 2 ** 127 * float(2 ** 8 - 1) / 2 ** 7
    return _core(x, 9, 8, max_norm, round, False)


_BLOCK_NAMES = {ElemFormat.fp8_e4m3: "MXFP8_E4M3", ElemFormat.fp8_e5m2: "MXFP8_E5M2", ElemFormat.fp6_e3m2: "MXFP6_E3M2",
                ElemFormat.fp6_e2m3: "MXFP6_E2M3", ElemFormat.fp4: "MXFP4"}


def block_quantize(x, fmt, axis=-1, block_size=32, scale_bits=8, round="even"):
    """OCP MX block quantization, dequantized output (_quantize_mx): the shared exponent and the saturating element
    step of block.ocp, then P * 2^shared_exp."""
    from ..block import ocp
    from ..block._driver import dequantize
    fmt = ElemFormat.from_str(fmt) if isinstance(fmt, str) else fmt
    if fmt not in _BLOCK_NAMES:
        raise NotImplementedError(f"mxq_b200: block_quantize has kernels for the OCP MX element formats, not {fmt}")
    P, X = ocp.quantize(x, _BLOCK_NAMES[fmt], axis=axis, block_size=block_size, rounding_mode=round,
                        scale_bits=scale_bits)
    return dequantize(P, X, axis=axis, block_size=block_size)
