"""mxq.lut — MX-Gemmini's look-up tables: a 4-bit index into a 16-entry table of element values per 2^G columns of
a K×n operand (mxq/lut/__init__.py).

    T = tables(P, fmt, group=G, max_iters=50)     P: K×n block codes; T: (n >> G) × 16, rows ascending
    I = pick(P, T, group=G)                        host pick: nearest entry, ties to the lower index
    I = finder(codes, T, fmt, group=G)             the chip's finder, from element codes
    P_lut = lookup(I, T, group=G)
"""
from .formats import FORMATS, SIZE, decode, encode, finder, values
from .kmeans import lookup, pick, tables

__all__ = ["FORMATS", "SIZE", "decode", "encode", "finder", "values", "tables", "pick", "lookup"]
