"""Pin the CPU oracle (oracle/mxq_oracle.c, oracle/lut_oracle.c) to the reference's own outputs: every golden
fixture written by tests/golden/make_golden.py is recomputed by the oracle and compared bit for bit (NaN-aware).
CPU only: this is what makes the oracle trustworthy as the checker for the CUDA kernels."""
import json

import numpy as np
import pytest

from _util import assert_bits, assert_bits_where, golden, nan_block_mask

FMT_EM = {(4, 3): "MXFP8_E4M3", (5, 2): "MXFP8_E5M2", (3, 2): "MXFP6_E3M2", (2, 3): "MXFP6_E2M3", (2, 1): "MXFP4"}


def _keys(g, prefix):
    return sorted(k for k in g if k.startswith(prefix))


# --------------------------------------------------------------------------------------------- elementwise
def test_float_em_f32(oracle):
    g = golden("elementwise")
    z = g["corpus"]
    ks = [k for k in _keys(g, "float_em/")]
    assert len(ks) == 2 * 3 * 12 + 3 * 5
    for k in ks:
        _, grid, mode, e, m = k.split("/")
        assert_bits(oracle.float_em(z, int(e), int(m), mode, grid), g[k], k)


def test_float_em_f64(oracle):
    g = golden("elementwise")
    z = g["corpus64"]
    for k in _keys(g, "float_em64/"):
        _, grid, mode, e, m = k.split("/")
        assert_bits(oracle.float_em(z, int(e), int(m), mode, grid), g[k], k)


def test_round_bits_int_bf16(oracle):
    g = golden("elementwise")
    for mode in ("ties_away", "rne", "truncate"):
        assert_bits(oracle.round_bits(g["round_bits/bits"], g["round_bits/keep"], mode), g[f"round_bits/{mode}"], mode)
        assert_bits(oracle.round_bits(g["round_bits/bits"], 7, mode), g[f"round_bits/{mode}/k7"], mode)
        assert_bits(oracle.round_int(g["round_int/in"], mode), g[f"round_int/{mode}"], mode)
        assert_bits(oracle.round_int(g["round_int/in"].astype(np.float64) * 1.5, mode), g[f"round_int64/{mode}"], mode)
    assert_bits(oracle.bf16(g["corpus"]), g["bf16"], "bf16")


def test_microsoft(oracle):
    g = golden("elementwise")
    z = g["corpus"]
    ks = _keys(g, "microsoft/")
    assert len(ks) == 30
    for k in ks:
        _, fmt, mode, sat = k.split("/")
        assert_bits(oracle.microsoft(z, fmt, mode, sat == "sat"), g[k], k)


def test_scale_rules(oracle):
    g = golden("elementwise")
    amax = g["amax"]
    for k in _keys(g, "scale/mxquant/"):
        assert_bits(oracle.scale_mxquant(amax, float(k.split("/")[2])), g[k], k)
    for k in _keys(g, "scale/ocp/"):
        _, _, emax, sb = k.split("/")
        assert_bits(oracle.scale_ocp(amax, int(emax), int(sb)), g[k], k)
    for k in _keys(g, "scale/ocp_below_top/"):
        _, _, emax, sb = k.split("/")
        assert_bits(oracle.scale_ocp(amax, int(emax) - 1, int(sb)), g[k], k)
    for k in _keys(g, "scale/ocp_no_clip/"):
        _, _, fmt, mode = k.split("/")
        assert_bits(oracle.scale_ocp_no_clip(amax, fmt, mode), g[k], k)


def test_arith(oracle):
    g = golden("elementwise")
    z = g["corpus"]
    for k in _keys(g, "truncate_significand/"):
        assert_bits(oracle.truncate_significand(z, int(k.split("/")[1])), g[k], k)
    for k in _keys(g, "flush_product/"):
        assert_bits(oracle.flush_product(z, int(k.split("/")[1])), g[k], k)
    for k in _keys(g, "saturate/"):
        _, lim, val = k.split("/")
        assert_bits(oracle.saturate(z, float(lim), float(val)), g[k], k)
    n = 0
    for k in _keys(g, "exact_add/"):
        parts = k.split("/")
        if len(parts) != 3:
            continue
        e, m = int(parts[1]), int(parts[2])
        assert_bits(oracle.exact_add(g[k + "/a"], g[k + "/b"], e, m), g[k], k)
        n += 1
    assert n == 14
    for k in _keys(g, "exact_add_g/"):
        parts = k.split("/")
        if len(parts) != 5:
            continue
        e, m, mode, grid = int(parts[1]), int(parts[2]), parts[3], parts[4]
        assert_bits(oracle.exact_add(g[k + "/a"], g[k + "/b"], e, m, mode, grid), g[k], k)


# ------------------------------------------------------------------------------------------------ block
def test_block_named(oracle):
    g = golden("block")
    V = g["V"]
    n = 0
    for fam in ("mxquant", "mxgemmini", "ocp"):
        for fmt in FMT_EM.values():
            for axis in (0, 1):
                P, X = oracle.block_quantize(V, fam, fmt, axis)
                keep = ~nan_block_mask(V, axis) if fam == "mxquant" else np.ones(V.shape, bool)
                assert_bits_where(P, g[f"{fam}/{fmt}/{axis}/P"], keep, f"{fam}/{fmt}/{axis}/P")
                assert_bits(X, g[f"{fam}/{fmt}/{axis}/X"], f"{fam}/{fmt}/{axis}/X")
                n += 1
    assert n == 30


def test_block_variants(oracle):
    g = golden("block")
    V = g["V"]
    for k in _keys(g, "mxgemmini_k/"):
        if not k.endswith("/P"):
            continue
        _, fmt, mode, fl, _ = k.split("/")
        P, X = oracle.block_quantize(V, "mxgemmini", fmt, 0, 32, mode, float(fl))
        assert_bits(P, g[k], k)
        assert_bits(X, g[k[:-1] + "X"], k)
    P, X = oracle.block_quantize(V, "mxgemmini", "MXFP4", 0, 32, "rne", via=(3, 1))
    assert_bits(P, g["mxgemmini_via/P"], "via P")
    assert_bits(X, g["mxgemmini_via/X"], "via X")
    for k in _keys(g, "ocp_p/"):
        if not k.endswith("/P"):
            continue
        _, fmt, pl, mode, _ = k.split("/")
        P, X = oracle.block_quantize(V, "ocp", fmt, 1, 32, mode, placement=pl)
        assert_bits(P, g[k], k)
        assert_bits(X, g[k[:-1] + "X"], k)
    for fmt in ("MXFP8_E4M3", "MXFP6_E3M2"):
        P, X = oracle.block_quantize(V, "ocp", fmt, 0, 32, "floor", scale_bits=5)
        assert_bits(P, g[f"ocp_sb/{fmt}/P"], fmt)
        assert_bits(X, g[f"ocp_sb/{fmt}/X"], fmt)
    P, X = oracle.block_quantize(V, "mxgemmini", "FP32", 0)
    assert_bits(P, g["fp32/P"], "fp32 P")
    assert_bits(X, g["fp32/X"], "fp32 X")


def test_block_odd_shapes(oracle):
    g = golden("block")
    V3 = g["V3"]
    for fam in ("mxquant", "mxgemmini", "ocp"):
        for axis in (0, 1, 2, -1):
            P, X = oracle.block_quantize(V3, fam, "MXFP8_E4M3", axis)
            keep = ~nan_block_mask(V3, axis) if fam == "mxquant" else np.ones(V3.shape, bool)
            assert_bits_where(P, g[f"odd/{fam}/{axis}/P"], keep, f"odd/{fam}/{axis}")
            assert_bits(X, g[f"odd/{fam}/{axis}/X"], f"odd/{fam}/{axis}")
        for bs in (16, 7):
            P, X = oracle.block_quantize(V3, fam, "MXFP6_E2M3", 1, bs)
            assert_bits(P, g[f"bs/{fam}/{bs}/P"], f"bs/{fam}/{bs}")
            assert_bits(X, g[f"bs/{fam}/{bs}/X"], f"bs/{fam}/{bs}")


# --------------------------------------------------------------------------------------------- reducers
def _arith(oracle, ar):
    if ar[0] == "mxg":
        return oracle.arith_mxgemmini(ar[1], ar[2], ar[3])
    return oracle.arith_mxquant(ar[1], ar[2])


def reducer_cases():
    g = golden("reducers")
    return sorted(json.loads(str(g["meta"])).items())


@pytest.mark.parametrize("name,case", reducer_cases(), ids=[n for n, _ in reducer_cases()])
def test_reducers(oracle, name, case):
    g = golden("reducers")
    ops = [g[f"{name}/{k}"] for k in ("P_A", "X_A", "P_B", "X_B")]
    red, ar, sched, size, kw = case["reducer"], case["arith"], case["schedule"], case["size"], case["kw"]
    sched = None if sched is None else [tuple(s) for s in sched]
    if red == "systolic":
        Y = oracle.systolic(*ops, _arith(oracle, ar), sched, size)
    elif red == "adder":
        Y = oracle.adder_tree(*ops, _arith(oracle, ar), sched, size)
    elif red == "anchor":
        Y = oracle.anchor_tree(*ops, _arith(oracle, ar), sched, size, **kw)
    else:
        Y = oracle.fp64_accum(*ops)
    assert_bits(Y, g[f"{name}/Y"], name)


def test_config1_full(oracle):
    """The PR1 workload at full size (256x512 output, K=512), MXGEMMINI / HW_FINAL."""
    g = golden("reducers")
    hw = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]
    ops = [g[f"config1/{k}"] for k in ("P_A", "X_A", "P_B", "X_B")]
    Y = oracle.systolic(*ops, oracle.arith_mxgemmini(), hw, 16)
    assert_bits(Y, g["config1/Y"], "config1")


# -------------------------------------------------------------------------------------------------- LUT
def test_lut_format_tables(oracle):
    g = golden("lut")
    for fmt in oracle.LUT_FORMATS:
        vals, fx, safe = oracle.lut_format_tables(fmt)
        assert_bits(vals, g[f"tables/{fmt}/vals"], fmt)
        assert_bits(fx, g[f"tables/{fmt}/fx"], fmt)
        assert_bits(safe, g[f"tables/{fmt}/safe"], fmt)


def test_lut_ops(oracle):
    g = golden("lut")
    for fmt in oracle.LUT_FORMATS:
        for G in (0, 1, 3):
            P = g[f"lut/{fmt}/{G}/P"]
            T = oracle.lut_tables(P, fmt, G, 50)
            assert_bits(T, g[f"lut/{fmt}/{G}/T"], f"tables {fmt} G{G}")
            assert_bits(oracle.lut_tables(P, fmt, G, 2), g[f"lut/{fmt}/{G}/T_it2"], f"tables it2 {fmt} G{G}")
            I = oracle.lut_pick(P, T, G)
            assert_bits(I, g[f"lut/{fmt}/{G}/I"], f"pick {fmt} G{G}")
            assert_bits(oracle.lut_lookup(I, T, G), g[f"lut/{fmt}/{G}/lookup"], f"lookup {fmt} G{G}")
            if f"lut/{fmt}/{G}/codes" in g:
                codes = g[f"lut/{fmt}/{G}/codes"]
                assert_bits(oracle.lut_encode(P, fmt), codes, f"encode {fmt}")
                assert_bits(oracle.lut_encode(T, fmt), g[f"lut/{fmt}/{G}/Tcodes"], f"encode T {fmt}")
                assert_bits(oracle.lut_finder(codes, T, fmt, G), g[f"lut/{fmt}/{G}/finder"], f"finder {fmt} G{G}")
        # negative codes count from the end (torch indexing in decode and finder)
        neg = g[f"lut/{fmt}/codes_neg"]
        assert_bits(oracle.lut_decode(neg, fmt), g[f"lut/{fmt}/decode_neg"], f"decode negative {fmt}")
        assert_bits(oracle.lut_finder(neg, g[f"lut/{fmt}/1/T"], fmt, 1), g[f"lut/{fmt}/finder_neg"],
                    f"finder negative {fmt}")
        # a code outside [-n, n) is an IndexError, raised before a table value that is no code is looked at
        bad = neg.copy()
        bad[0, 0] = 1 << 20
        Tbad = g[f"lut/{fmt}/1/T"].copy()
        Tbad[0, 0] = np.float32(0.1)
        with pytest.raises(IndexError):
            oracle.lut_finder(bad, Tbad, fmt, 1)
        with pytest.raises(ValueError):
            oracle.lut_finder(neg, Tbad, fmt, 1)
        with pytest.raises(IndexError):
            oracle.lut_decode(bad, fmt)


def test_lut_block(oracle):
    g = golden("lut")
    V = g["V"]
    for fmt in oracle.LUT_FORMATS:
        for G in (0, 1, 3):
            for axis in (0, 1):
                P, X = oracle.lut_block_quantize(V, fmt, axis, 32, "rne", 2.0 ** -23, G, 50)
                assert_bits(P, g[f"blut/{fmt}/{G}/{axis}/P"], f"blut {fmt} {G} {axis}")
                assert_bits(X, g[f"blut/{fmt}/{G}/{axis}/X"], f"blut {fmt} {G} {axis}")
