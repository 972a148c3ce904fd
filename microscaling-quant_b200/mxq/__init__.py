"""mxq — microscaling (MX) quantization and MX-Gemmini matmul emulation, on B200 (sm_100a) CUDA kernels.

The same API as the reference package (chloe-wong/microscaling-quant): block quantization in two steps (scale
factor, element quantization), MX-Gemmini's LUT codebooks, and the emulated matmuls (systolic / anchor tree / adder
tree) with their Arithmetics and schedules, plus the nn layers that put them into a model. Every computing call is
a kernel of libmxq_b200.so (microscaling-quant_b200/csrc, C ABI in include/mxq_b200.h); there is no CPU path.
"""
__version__ = "0.1.0"

from . import rounding, arith, schedule, scale_factor, element_quant, lut, block, matmul, scheme, nn, microxcaling, shard
from .block import BLOCK
from ._fp64_accum import fp64_accum
from .element_quant.formats import Format
from .scheme import Scheme

__all__ = ["microxcaling", "rounding", "arith", "schedule", "scale_factor", "element_quant", "lut", "block", "matmul",
           "scheme", "nn", "BLOCK", "Format", "Scheme", "fp64_accum"]
