"""mxq.block — block quantization: step 1 (scale_factor) and step 2 (element_quant) composed.

    P, X = block.compose(V, scale=f, elem=g, axis=0, block_size=BLOCK)   any pair
    P, X = block.<name>.quantize(V, fmt, axis=0, block_size=BLOCK)     mxquant | mxgemmini | ocp | lut
    V_hat = block.<name>.dequantize(P, X, axis=0)                      = P * expand(X)

The named quantizers run as one fused CUDA kernel each (read V once, write P and X once).
"""
from ._driver import BLOCK, compose, dequantize, dequantize_packed, unpack
from . import mxquant, mxgemmini, ocp, lut

__all__ = ["BLOCK", "compose", "dequantize", "mxquant", "mxgemmini", "ocp", "lut", "unpack", "dequantize_packed"]
