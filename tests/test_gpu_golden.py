"""The CUDA kernels, through the public mxq API, against every golden fixture of the reference: the same checks
that pin the CPU oracle (tests/test_oracle_golden.py), run with the product behind the oracle's names."""
import json

import numpy as np
import pytest

import test_oracle_golden as g
from _util import assert_bits, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prod():
    import mxq_adapter
    return mxq_adapter


@pytest.mark.parametrize("check", [g.test_float_em_f32, g.test_float_em_f64, g.test_round_bits_int_bf16,
                                   g.test_microsoft, g.test_scale_rules, g.test_arith],
                         ids=lambda f: f.__name__[5:])
def test_elementwise(prod, check):
    check(prod)


@pytest.mark.parametrize("check", [g.test_block_named, g.test_block_variants, g.test_block_odd_shapes],
                         ids=lambda f: f.__name__[5:])
def test_block(prod, check):
    check(prod)


@pytest.mark.parametrize("name,case", g.reducer_cases(), ids=[n for n, _ in g.reducer_cases()])
def test_reducers(prod, name, case):
    g.test_reducers(prod, name, case)


def test_config1(prod):
    """The PR1 workload end to end on the GPU: the seeded x (256x512) and W (512x512) regenerated with torch's CPU
    generator, quantized by block.mxgemmini on the device, reduced by systolic MXGEMMINI / HW_FINAL; every code,
    scale and output equal to the reference's."""
    import torch
    import mxq
    gd = golden("reducers")
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(256, 512, generator=gen)
    W = torch.randn(512, 512, generator=gen)
    assert float(x.double().sum()) == float(gd["config1/x_sum"]) and float(W.double().sum()) == float(gd["config1/W_sum"])
    P_A, X_A = mxq.block.mxgemmini.quantize(x.t().cuda(), "MXFP8_E4M3", axis=0)
    P_B, X_B = mxq.block.mxgemmini.quantize(W.t().cuda(), "MXFP8_E4M3", axis=0)
    for name, t in (("P_A", P_A), ("X_A", X_A), ("P_B", P_B), ("X_B", X_B)):
        assert_bits(t, gd[f"config1/{name}"], name)
    Y = mxq.matmul.systolic(P_A, X_A, P_B, X_B, mxq.matmul.MXGEMMINI(), mxq.schedule.HW_FINAL)
    assert_bits(Y, gd["config1/Y"], "config1 Y")


@pytest.mark.parametrize("check", [g.test_lut_ops, g.test_lut_block], ids=lambda f: f.__name__[5:])
def test_lut(prod, check):
    check(prod)
