"""The CUDA kernels' element math (numerics.cuh), compiled for the host with g++, checked without a GPU:
against every elementwise golden fixture of the reference, against the CPU oracle on large random corpora, and
floor(log2 x) exhaustively over all positive float32 against the torch-derived thresholds."""
import ctypes
import json
import os
import subprocess

import numpy as np
import pytest

from _util import GOLDEN, assert_bits, golden

HERE = os.path.dirname(os.path.abspath(__file__))
SHIM = os.path.join(HERE, "host", "numerics_shim.cpp")
LIB = os.path.join(HERE, "host", "_build", "libnumerics_shim.so")


@pytest.fixture(scope="module")
def shim():
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    src_mtime = max(os.path.getmtime(SHIM), os.path.getmtime(
        os.path.join(HERE, "..", "microscaling-quant_b200", "csrc", "numerics.cuh")))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < src_mtime:
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
                        "-o", LIB, SHIM], check=True)
    return ctypes.CDLL(LIB)


class _Proxy:
    """Routes the oracle's o_* calls to the shim's h_* twins."""

    def __init__(self, cdll):
        self.c = cdll

    def __getattr__(self, name):
        return getattr(self.c, "h_" + name[2:])


@pytest.fixture()
def host(oracle, shim):
    saved = oracle._lib
    oracle._lib = _Proxy(shim)
    yield oracle
    oracle._lib = saved


def test_host_numerics_golden(host):
    """The same fixtures tests/test_oracle_golden.py pins the oracle with, through numerics.cuh."""
    import test_oracle_golden as t
    for fn in (t.test_float_em_f32, t.test_float_em_f64, t.test_round_bits_int_bf16, t.test_microsoft,
               t.test_scale_rules, t.test_arith):
        fn(host)


def test_host_numerics_random_vs_oracle(oracle, shim):
    """Random bit patterns and grid-valued operands: numerics.cuh and the oracle agree everywhere."""
    rng = np.random.default_rng(11)
    z = rng.integers(0, 2 ** 32, 400000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    ref = {}
    for grid in ("qtorch", "ieee", "ocp"):
        ems = [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)] if grid == "ocp" else [(4, 4), (4, 6), (8, 7), (5, 10), (3, 3)]
        for mode in ("ties_away", "rne", "truncate"):
            for e, m in ems:
                ref[(grid, mode, e, m)] = oracle.float_em(z, e, m, mode, grid)
    saved = oracle._lib
    oracle._lib = _Proxy(shim)
    try:
        for (grid, mode, e, m), want in ref.items():
            assert_bits(oracle.float_em(z, e, m, mode, grid), want, f"{grid}/{mode}/{e}/{m}")
    finally:
        oracle._lib = saved
    for fmt in ("MXFP8_E4M3", "MXFP6_E2M3", "MXFP4"):
        for mode in ("nearest", "even", "floor"):
            want = oracle.microsoft(z, fmt, mode, True)
            oracle._lib = _Proxy(shim)
            try:
                assert_bits(oracle.microsoft(z, fmt, mode, True), want, f"ms/{fmt}/{mode}")
            finally:
                oracle._lib = saved


def test_log2_thresholds_match_torch(shim):
    """floor_log2_rn's thresholds equal the ones measured from torch.floor(torch.log2(x)) over all float32."""
    want = json.load(open(os.path.join(GOLDEN, "log2_floor.json")))["thresholds"]
    out = np.zeros(278, np.uint32)
    shim.h_log2_thresholds(out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    got = {k: int(out[k + 149]) for k in range(-149, 129)}
    assert {int(k): v for k, v in want.items()} == got


def test_log2_exhaustive_vs_libm(shim):
    """floor_log2_rn against floor((float)log2((double)x)) on every positive finite float32."""
    f = shim.h_log2_mismatches
    f.restype = ctypes.c_int64
    from concurrent.futures import ThreadPoolExecutor
    cuts = np.linspace(1, 0x7F800000, 9).astype(np.int64)
    with ThreadPoolExecutor(8) as ex:
        bad = sum(ex.map(lambda i: f(ctypes.c_uint32(int(cuts[i])), ctypes.c_uint32(int(cuts[i + 1]))), range(8)))
    assert bad == 0


@pytest.mark.parametrize("which", [0, 1], ids=["ocp_grid", "microsoft"])
def test_fast_forms_match_general(shim, which):
    """The block quantizer's bit-level element forms (q_ocp_bits, q_microsoft_sat) equal the general functions
    on a dense stride through all 2^32 float32 patterns, for every OCP format and rounding mode."""
    f = shim.h_fast_forms_mismatches
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int]
    from concurrent.futures import ThreadPoolExecutor
    stride, chunk = 4099, 1 << 29                      # 8 chunks of the 2^32 patterns per (format, mode)
    jobs = [(lo, e, m, mode) for (e, m) in [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)] for mode in range(3)
            for lo in range(0, 1 << 32, chunk)]
    with ThreadPoolExecutor(8) as ex:
        bad = sum(ex.map(lambda j: f(j[0], j[0] + chunk, stride, which, j[1], j[2], j[3]), jobs))
    assert bad == 0


def test_microsoft_ocp_form_matches_general(shim):
    """q_microsoft_ocp (the TMA quantizer's ocp element step) equals q_microsoft on a dense stride through all
    2^32 patterns for every OCP format and rounding mode; the exhaustive run is in the repository's history."""
    f = shim.h_ms_ocp_mismatches
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    from concurrent.futures import ThreadPoolExecutor
    stride, chunk = 4099, 1 << 29
    jobs = [(lo, e, m, mode) for (e, m) in [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)] for mode in range(3)
            for lo in range(0, 1 << 32, chunk)]
    with ThreadPoolExecutor(8) as ex:
        bad = sum(ex.map(lambda j: f(j[0], j[0] + chunk, stride, j[1], j[2], j[3]), jobs))
    assert bad == 0


@pytest.mark.parametrize("which", [0, 1], ids=["ocp_grid", "microsoft"])
def test_small_forms_match_general(shim, which):
    """The clean-tile element forms (q_ocp_small, q_microsoft_ocp_small: rounding by one float add at the step's
    magic constant) equal q_ocp_bits / q_microsoft_ocp_core on every pattern with |x| < 2^17 on a dense stride, for
    every OCP format and rounding mode, including the one value where microxcaling's even is not RNE."""
    f = shim.h_small_forms_mismatches
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int]
    from concurrent.futures import ThreadPoolExecutor
    stride, chunk = 1021, 1 << 29
    jobs = [(lo, e, m, mode) for (e, m) in [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)] for mode in range(3)
            for lo in range(0, 1 << 32, chunk)]
    with ThreadPoolExecutor(8) as ex:
        bad = sum(ex.map(lambda j: f(j[0], j[0] + chunk, stride, which, j[1], j[2], j[3]), jobs))
    assert bad == 0
    # the exception itself: (0.5 - 2^-25) * 2^(min_exp - m) in every format, both signs, with its neighbours
    for (e, m) in [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)]:
        min_exp = 2 - (1 << (e - 1))
        star = ((min_exp + 127 - m - 2) << 23) | 0x7FFFFF
        for v in (star - 1, star, star + 1, star | 0x80000000):
            for mode in range(3):
                assert f(v, v + 1, 1, which, e, m, mode) == 0


def test_ieee_small_matches_general(shim):
    """q_ieee_small (the via pre-rounding of clean tiles: one float add at the step's magic constant) equals
    q_ieee_f on patterns with |x| < 2^17, on a stride, for float(e, m) with e 1..7 and m from 1 to 21, every mode."""
    f = shim.h_ieee_small_mismatches
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    from concurrent.futures import ThreadPoolExecutor
    fmts = [(e, m) for e in range(1, 8) for m in (1, 2, 3, 5, 10, 21)]
    jobs = [(lo, e, m, mode) for (e, m) in fmts for mode in range(3) for lo in range(0, 1 << 32, 1 << 30)]
    with ThreadPoolExecutor(8) as ex:
        bad = sum(ex.map(lambda j: f(j[0], j[0] + (1 << 30), 65537, j[1], j[2], j[3]), jobs))
    assert bad == 0


def test_microsoft_even_is_not_rint(shim):
    """Regression: the reference's even rounding rounds |t| + 0.5 in float32 before the floor, so 2^-10 (1 - 2^-24)
    in MXFP8_E4M3 (t = 0.5 - 2^-25 after clipping) becomes 2^-9, where round-half-even would give 0."""
    f = shim.h_ms_ocp_mismatches
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    for base in (0x3A7FFFFF, 0xBA7FFFFF):
        for e, m in [(4, 3), (5, 2)]:
            assert f(base - 64, base + 64, 1, e, m, 2) == 0
