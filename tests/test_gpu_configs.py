"""Every BASELINE config at the size and on the inputs the bench runs, against the CPU oracle (oracle/, pinned to the
reference's own outputs by tests/test_oracle_golden.py), bit for bit:

  config 2  the bench's seeded 8192 x 8192 matrix (bench.synthetic(8192, 8192, 1000) on the device), all 30 runs of
            the sweep, codes P and scales X, the whole matrix
  config 3  the bench's 4096 x 4096 operands, quantized to MXFP8_E4M3 and MXFP6_E2M3 (checked whole), the full
            4096 x 4096 Y of each of the four reducers computed on the GPU (so the 64 x 128 CTA tiles and K = 4096, 128
            k-blocks, run as they do in the bench) and 8 output tiles of 64 x 64 at full K compared with the oracle
  config 4  the bench's 4096 x 4096 LUT operand: block.lut.quantize for MXFP6_E3M2 and MXFP8_E4M3 x group 1 and 3
            (P_lut and X whole), and lut.tables / pick / encode / finder on the MXFP6_E3M2 codes
  config 5  the full-size patched Llama (16 layers, hidden 2048, FFN 5632, 16 heads x 128, vocab 32000) on a
            16-token prefix: every MXLinear of layers 0 and 15 on its captured input against the oracle's quantize +
            systolic (a 256-column slice of each output), and the batch-row independence the batch split relies on
            (each row's logits from the batched forward against that row alone, 1e-6 relative).
"""
import os
import sys
from functools import partial

import numpy as np
import pytest
import torch

from _util import assert_bits

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

HW = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]
LEVELS = [(4, 4), (4, 5), (4, 6), (8, 7)]
FAMILIES = ("mxquant", "mxgemmini", "ocp")
FORMATS = ("MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4")


def test_config2_full_sweep(oracle):
    import bench
    from mxq import block
    quant = {"mxquant": block.mxquant.quantize, "mxgemmini": block.mxgemmini.quantize, "ocp": block.ocp.quantize}
    V = bench.synthetic(8192, 8192, 1000, torch.device("cuda", 0))
    Vh = V.cpu().numpy()
    for f in FAMILIES:
        for fmt in FORMATS:
            for ax in (0, 1):
                P, X = quant[f](V, fmt, axis=ax)
                Po, Xo = oracle.block_quantize(Vh, f, fmt, ax)
                assert_bits(P.cpu().numpy(), Po, f"{f} {fmt} axis {ax} P")
                assert_bits(X.cpu().numpy(), Xo, f"{f} {fmt} axis {ax} X")
                del P, X, Po, Xo


def _tiles():
    """8 output tiles (row offset, column offset) of 64 x 64 spread over a 4096 x 4096 Y, off the 512 grid."""
    return [(i * 512 + 64 * (i % 3), ((5 * i + 2) % 8) * 512 + 64 * (i % 5)) for i in range(8)]


@pytest.mark.parametrize("fmt", ["MXFP8_E4M3", "MXFP6_E2M3"])
def test_config3_reducers_full_k(oracle, fmt):
    import bench
    from mxq import block, matmul, schedule

    class _R:
        dev = torch.device("cuda", 0)
        torch = torch
    A, B = bench.gemm_operands(_R())
    P_A, X_A = block.mxgemmini.quantize(A, fmt, axis=0)
    P_B, X_B = block.mxgemmini.quantize(B, fmt, axis=0)
    ops = [t.cpu().numpy() for t in (P_A, X_A, P_B, X_B)]
    oPA, oXA = oracle.block_quantize(A.cpu().numpy(), "mxgemmini", fmt, 0)
    oPB, oXB = oracle.block_quantize(B.cpu().numpy(), "mxgemmini", fmt, 0)
    for name, got, want in (("P_A", ops[0], oPA), ("X_A", ops[1], oXA), ("P_B", ops[2], oPB), ("X_B", ops[3], oXB)):
        assert_bits(got, want, f"config 3 {fmt} {name}")
    arith = matmul.MXGEMMINI()
    cases = {
        "systolic MXGEMMINI": (lambda: matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL),
                               lambda a, b, c, d: oracle.systolic(a, b, c, d, oracle.arith_mxgemmini(), HW)),
        "systolic MXQUANT(4,3)": (lambda: matmul.systolic(P_A, X_A, P_B, X_B, matmul.MXQUANT(4, 3), schedule.HW_FINAL),
                                  lambda a, b, c, d: oracle.systolic(a, b, c, d, oracle.arith_mxquant(4, 3), HW)),
        "adder_tree": (lambda: matmul.adder_tree(P_A, X_A, P_B, X_B, arith, LEVELS),
                       lambda a, b, c, d: oracle.adder_tree(a, b, c, d, oracle.arith_mxgemmini(), LEVELS)),
        "anchor_tree": (lambda: matmul.anchor_tree(P_A, X_A, P_B, X_B, arith),
                        lambda a, b, c, d: oracle.anchor_tree(a, b, c, d, oracle.arith_mxgemmini())),
    }
    for name, (gpu, cpu) in cases.items():
        Y = gpu().cpu().numpy()
        assert Y.shape == (4096, 4096)
        for r, c in _tiles():
            want = cpu(ops[0][:, r:r + 64], ops[1][:, r:r + 64], ops[2][:, c:c + 64], ops[3][:, c:c + 64])
            assert_bits(Y[r:r + 64, c:c + 64], want, f"config 3 {fmt} {name} tile ({r}, {c})")


def test_config4_lut_full_size(oracle):
    import bench
    from mxq import block, lut

    class _R:
        dev = torch.device("cuda", 0)
        torch = torch
    V = bench.config4_operand(_R(), 13)
    Vh = V.cpu().numpy()
    for fmt in ("MXFP6_E3M2", "MXFP8_E4M3"):
        for G in (1, 3):
            P, X = block.lut.quantize(V, fmt, 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23, group=G,
                                      max_iters=50)
            Po, Xo = oracle.lut_block_quantize(Vh, fmt, 0, 32, "rne", 2.0 ** -23, G, 50)
            assert_bits(P.cpu().numpy(), Po, f"block.lut {fmt} G={G} P")
            assert_bits(X.cpu().numpy(), Xo, f"block.lut {fmt} G={G} X")
    P4 = block.mxgemmini.quantize(V, "MXFP6_E3M2", 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
    P4h = P4.cpu().numpy()
    T = lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=50)
    To = oracle.lut_tables(P4h, "MXFP6_E3M2", 1, 50)
    assert_bits(T.cpu().numpy(), To, "lut.tables")
    assert_bits(lut.pick(P4, T, group=1).cpu().numpy(), oracle.lut_pick(P4h, To, 1), "lut.pick")
    C = lut.encode(P4, "MXFP6_E3M2")
    Co = oracle.lut_encode(P4h, "MXFP6_E3M2")
    assert_bits(C.cpu().numpy(), Co, "lut.encode")
    assert_bits(lut.finder(C, T, "MXFP6_E3M2", group=1).cpu().numpy(), oracle.lut_finder(Co, To, "MXFP6_E3M2", 1),
                "lut.finder")


def test_config5_full_size_layers(oracle):
    import bench

    class _R:
        dev = torch.device("cuda", 0)
        torch = torch
    model, handle = bench.llama(_R())
    captured = {}

    def hook(name):
        def f(mod, inp, out):
            captured[name] = (inp[0].detach(), out.detach())
        return f
    for name, mod in model.named_modules():
        if type(mod).__name__ == "MXLinear" and (".layers.0." in name or ".layers.15." in name):
            mod.register_forward_hook(hook(name))
    ids = torch.randint(0, 32000, (2, 16), generator=torch.Generator(device="cuda").manual_seed(14), device="cuda")
    with torch.no_grad():
        batched = model(ids).logits
        rows = [model(ids[b:b + 1]).logits for b in range(2)]
    assert len(captured) == 14
    mods = dict(model.named_modules())
    for name, (x, y) in captured.items():
        W = mods[name].weight.detach().float()
        xt = x.reshape(-1, x.shape[-1]).float().t().contiguous().cpu().numpy()    # A = xᵀ: K x tokens
        Wt = W.t().contiguous().cpu().numpy()                                     # B = Wᵀ: K x out
        cols = slice(0, 256)
        PA, XA = oracle.block_quantize(xt, "mxgemmini", "MXFP8_E4M3", 0)
        PB, XB = oracle.block_quantize(np.ascontiguousarray(Wt[:, cols]), "mxgemmini", "MXFP8_E4M3", 0)
        want = oracle.systolic(PA, XA, PB, XB, oracle.arith_mxgemmini(), HW)
        got = y.reshape(-1, y.shape[-1])[:, cols].float().cpu().numpy()
        assert_bits(got, want, f"config 5 {name}")
    for b in range(2):
        want = rows[b][0].double()
        rel = float((batched[b].double() - want).abs().max() / want.abs().max())
        assert rel <= 1e-6, f"batch row {b}: {rel}"
    handle.revert()
    del model
    torch.cuda.empty_cache()
