"""mxq.element_quant — step 2 of block quantization: snap scaled values onto a format's codes.

    formats     the format table (name -> e, m, emax, max_norm)
    float_em    float(e, m) on the qtorch 0.2.0, ieee or OCP grid
    microsoft   the microxcaling element step (the OCP reference block algorithm's choice)
"""
from . import formats, float_em, microsoft

__all__ = ["formats", "float_em", "microsoft"]
