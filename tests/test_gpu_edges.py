"""Empty and ragged inputs through the public API on the GPU, against the oracle: block quantizers whose block axis
or whole tensor is empty, reducers with K = 0 (the output stays zero), M = 0 or N = 0, ragged K, M, N that leave
partial blocks, reductions and tiles; LUT fits of an operand with no rows (every group's table is padding only) and
block.lut of an empty operand."""
import numpy as np
import pytest

import mxq_adapter as prod
from _util import assert_bits

pytestmark = pytest.mark.gpu

HW = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]
LEVELS = [(4, 4), (4, 5), (4, 6), (8, 7)]


@pytest.mark.parametrize("shape,axis", [((0, 64), 0), ((64, 0), 1), ((5, 0, 3), 1), ((0, 3, 7), 0)])
def test_block_empty(oracle, shape, axis):
    V = np.zeros(shape, np.float32)
    for family in ("mxquant", "mxgemmini", "ocp"):
        P, X = prod.block_quantize(V, family, "MXFP8_E4M3", axis)
        Po, Xo = oracle.block_quantize(V, family, "MXFP8_E4M3", axis)
        assert P.shape == Po.shape and X.shape == Xo.shape, (family, P.shape, X.shape, Po.shape, Xo.shape)


@pytest.mark.parametrize("K,M,N", [(0, 4, 8), (32, 0, 4), (32, 4, 0), (7, 3, 5), (33, 5, 6), (70, 9, 130)])
def test_reducers_ragged(oracle, K, M, N):
    rng = np.random.default_rng(K * 100 + M * 10 + N)
    A = rng.standard_normal((K, M)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    P_A, X_A = oracle.block_quantize(A, "mxgemmini", "MXFP8_E4M3", 0)
    P_B, X_B = oracle.block_quantize(B, "mxgemmini", "MXFP8_E4M3", 0)
    ops = (P_A, X_A, P_B, X_B)
    cases = [
        ("systolic mxgemmini", prod.systolic(*ops, prod.arith_mxgemmini(), HW),
         oracle.systolic(*ops, oracle.arith_mxgemmini(), HW)),
        ("systolic mxquant", prod.systolic(*ops, prod.arith_mxquant(4, 3), HW),
         oracle.systolic(*ops, oracle.arith_mxquant(4, 3), HW)),
        ("adder", prod.adder_tree(*ops, prod.arith_mxgemmini(), LEVELS),
         oracle.adder_tree(*ops, oracle.arith_mxgemmini(), LEVELS)),
        ("anchor", prod.anchor_tree(*ops, prod.arith_mxgemmini()), oracle.anchor_tree(*ops, oracle.arith_mxgemmini())),
        ("fp64_accum", prod.fp64_accum(*ops), oracle.fp64_accum(*ops)),
    ]
    for what, got, want in cases:
        assert got.shape == (M, N), (what, got.shape)
        assert_bits(got, want, what)
        if K == 0:
            assert not np.any(got.view(np.uint32)), what          # +0 everywhere


def test_lut_no_rows(oracle):
    P = np.zeros((0, 8), np.float32)
    for fmt in ("MXFP6_E3M2", "MXFP8_E4M3"):
        T = prod.lut_tables(P, fmt, 1, 50)
        assert_bits(T, oracle.lut_tables(P, fmt, 1, 50), f"tables {fmt}")
        assert prod.lut_pick(P, T, 1).shape == (0, 8)
        assert prod.lut_finder(np.zeros((0, 8), np.int64), T, fmt, 1).shape == (0, 8)
        V = np.zeros((0, 64), np.float32)
        Pl, X = prod.lut_block_quantize(V, fmt, 0, 32, "rne", 2.0 ** -23, 1, 50)
        Plo, Xo = oracle.lut_block_quantize(V, fmt, 0, 32, "rne", 2.0 ** -23, 1, 50)
        assert Pl.shape == Plo.shape and X.shape == Xo.shape


@pytest.mark.parametrize("fmt", ["MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E4M3", "MXFP8_E5M2"])
def test_lut_block_bad_values(oracle, fmt):
    """block.lut of an operand holding a NaN or an Inf: the oracle refuses it (a code that is not a value of the
    format reaches the table fit) and so does the product, with the same ValueError, for every group size and both
    axes, with the bad value in one panel of several; the next call on clean data is still bit for bit."""
    rng = np.random.default_rng(7)
    K, n = 256, 160
    V = (rng.standard_normal((K, n)) * 2.0 ** rng.uniform(-4, 4, (1, n))).astype(np.float32)
    for bad in (np.nan, np.inf):
        Vb = V.copy()
        Vb[100, 70] = bad
        for G in (0, 1, 3):
            for axis in (0, 1):
                with pytest.raises(ValueError):
                    oracle.lut_block_quantize(Vb, fmt, axis, 32, "rne", 2.0 ** -23, G, 50)
                with pytest.raises(ValueError, match="not a"):
                    prod.lut_block_quantize(Vb, fmt, axis, 32, "rne", 2.0 ** -23, G, 50)
    for G in (1, 3):
        P, X = prod.lut_block_quantize(V, fmt, 0, 32, "rne", 2.0 ** -23, G, 50)
        Po, Xo = oracle.lut_block_quantize(V, fmt, 0, 32, "rne", 2.0 ** -23, G, 50)
        assert_bits(P, Po, f"block.lut {fmt} G{G} after a refused call")
        assert_bits(X, Xo, f"block.lut X {fmt} G{G} after a refused call")
