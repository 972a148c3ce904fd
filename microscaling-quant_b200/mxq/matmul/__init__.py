"""mxq.matmul — the array dataflows, Y = Aᵀ·B from codes and scales in the order the hardware sums them.

    Y = systolic(P_A, X_A, P_B, X_B, arith, schedule, size=16)       the PE column
    Y = anchor_tree(P_A, X_A, P_B, X_B, arith, schedule=None, size=16, *, width, bits, drop, headroom, emin)
    Y = adder_tree(P_A, X_A, P_B, X_B, arith, schedule, size=16)     a float(e, m) per tree level

A: K×M, B: K×N, X: one row of scales per block of K, Y: M×N float32. MXQUANT(prod_e, prod_m) and MXGEMMINI() are
the two Arithmetics (the rounding at each stage); each reducer is one CUDA kernel.
"""
from ._arithmetic import Arithmetic, MXQUANT, MXGEMMINI, compiled
from ._systolic import systolic
from ._anchor import anchor_tree
from ._adder import adder_tree
from ..schedule import HW_FINAL

__all__ = ["Arithmetic", "MXQUANT", "MXGEMMINI", "compiled", "systolic", "anchor_tree", "adder_tree", "HW_FINAL"]
