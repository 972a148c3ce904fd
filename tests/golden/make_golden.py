"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation
(chloe-wong/microscaling-quant, imported from its checkout) on seeded inputs.

    python tests/golden/make_golden.py [--reference PATH] [--only NAME ...]

The reference's package is also called `mxq`, so this script re-executes itself in a child process whose
PYTHONPATH holds only the reference checkout, and refuses to run if `mxq` resolves anywhere else. The fixtures
are the reference's own outputs; tests/test_oracle_golden.py checks the CPU oracle against them and the GPU
tests check the CUDA kernels against them directly. Nothing at test time reads the reference checkout.

Fixtures (all numpy .npz, float32 results compared bit for bit, NaN positions only for NaN):
    log2_floor.json   torch.floor(torch.log2(x)) thresholds over every positive float32 (exhaustive scan)
    elementwise.npz   rounding, float_em (3 grids x 3 modes), microxcaling element step, scale rules, arith
    block.npz         block.mxquant / mxgemmini / ocp / compose variants on a config-2-like matrix
    reducers.npz      systolic / anchor_tree / adder_tree / fp64_accum variants, and the full config-1 output
    lut.npz           lut.tables / pick / lookup / finder / encode / values and block.lut.quantize
    nn.npz            Scheme.matmul, MXLinear.forward and attend on small shapes
    model.npz         a small random-init Llama patched as config 5: logits, and every MXLinear's input / output
    api.npz           the rounding modules, block.compose with the reference's own steps and the blocking helpers,
                      schedule.load / fixed, the vector ops and vector="bf16" through patch, attend on decode / GQA /
                      multi-chunk causal shapes, patch's tables and errors, mxq.nn.torchao.MXQConfig
"""
import argparse
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))


# ------------------------------------------------------------------------------------------ corpora
def hard_corpus(np, n_random=3000, seed=1234):
    """float32 values that exercise every branch: specials, subnormals, binade edges, the ulps below a binade
    where log2 rounds up, rounding ties at 1..11 kept bits, and random bit patterns / magnitudes."""
    rng = np.random.default_rng(seed)
    u = []
    u += [0x00000000, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0xffc00000, 0x7fa00001, 0xffe12345,
          0x00000001, 0x80000001, 0x007fffff, 0x807fffff, 0x00800000, 0x80800000, 0x7f7fffff, 0xff7fffff,
          0x00400000, 0x006ce3ee, 0x00000003, 0x7f7fffd4, 0x7f7fffd3]
    for k in list(range(-149, 128, 3)) + list(range(-10, 12)):
        base = (k + 127) << 23 if k >= -126 else (1 << (k + 149))
        for d in (-45, -44, -43, -23, -22, -12, -11, -6, -5, -3, -2, -1, 0, 1, 2):
            b = base + d
            if 0 < b < 0x7f800000:
                u += [b, b | 0x80000000]
    for k in range(-20, 20):
        for m in range(1, 12):
            for j in (0, 1, 5):
                v = np.float32(2.0 ** k * (1 + (2 * j + 1) / 2 ** (m + 1)))
                u += [int(v.view(np.uint32)), int((-v).view(np.uint32))]
    u += [int(x) for x in rng.integers(0, 2 ** 32, n_random, dtype=np.uint64)]
    mags = rng.standard_normal(n_random) * 2.0 ** rng.uniform(-30, 30, n_random)
    u += [int(x) for x in mags.astype(np.float32).view(np.uint32)]
    small = rng.standard_normal(n_random) * 2.0 ** rng.integers(-12, 4, n_random)
    u += [int(x) for x in small.astype(np.float32).view(np.uint32)]
    return np.array(u, dtype=np.uint64).astype(np.uint32).view(np.float32)


def grid_values(np, torch, float_em, e, m, n, seed):
    """n values on the float(e, m) ieee grid (lane accumulator values), mixed magnitudes, both signs, zeros."""
    rng = np.random.default_rng(seed)
    b = (1 << (e - 1)) - 1
    lo, hi = -b - m - 2, b + 1
    x = rng.standard_normal(n) * 2.0 ** rng.integers(lo, hi, n)
    x[rng.random(n) < 0.03] = 0.0
    t = torch.tensor(x, dtype=torch.float32)
    q = float_em.quantize(t, e, m, rounding_mode="rne", grid="ieee")
    return q.numpy()


# ---------------------------------------------------------------------------------------------- child
def child(only):
    import numpy as np
    import torch
    import mxq
    ref = os.environ["MXQ_REFERENCE"]
    if not os.path.abspath(mxq.__file__).startswith(os.path.abspath(ref)):
        raise SystemExit(f"refusing: mxq resolves to {mxq.__file__}, not the reference at {ref}")
    torch.set_num_threads(os.cpu_count() or 1)
    from mxq import arith, block, lut, matmul, rounding, scale_factor, schedule
    from mxq.element_quant import float_em, microsoft
    from mxq._fp64_accum import fp64_accum

    def T(a, dtype=torch.float32):
        return torch.tensor(np.asarray(a)).to(dtype)

    def N(t):
        return t.detach().cpu().numpy()

    def want(name):
        return not only or name in only

    # --------------------------------------------------------------------------------- log2 thresholds
    if want("log2"):
        t0 = time.time()
        thr = {}
        prev = None
        CH = 1 << 26
        for start in range(1, 0x7F800000, CH):
            end = min(start + CH, 0x7F800000)
            x = torch.arange(start, end, dtype=torch.int64).to(torch.int32).view(torch.float32)
            f = torch.floor(torch.log2(x))
            if prev is None:
                thr[int(f[0])] = start
            elif f[0] != prev:
                thr[int(f[0])] = start
            d = torch.nonzero(f[1:] != f[:-1]).squeeze(1)
            for i in d.tolist():
                thr[int(f[i + 1])] = start + i + 1
            prev = f[-1].item()
        json.dump({"torch": torch.__version__, "thresholds": {str(k): v for k, v in sorted(thr.items())}},
                  open(os.path.join(HERE, "log2_floor.json"), "w"), indent=0)
        print(f"log2_floor.json: {len(thr)} thresholds, {time.time() - t0:.1f}s", flush=True)

    # ------------------------------------------------------------------------------------- elementwise
    if want("elementwise"):
        out = {}
        z = hard_corpus(np)
        out["corpus"] = z
        zt = T(z)
        EM = [(2, 1), (3, 2), (4, 3), (4, 4), (4, 6), (5, 2), (5, 10), (7, 10), (8, 7), (8, 10), (8, 23), (6, 17)]
        for grid in ("qtorch", "ieee"):
            for mode in rounding.MODES:
                for e, m in EM:
                    out[f"float_em/{grid}/{mode}/{e}/{m}"] = N(float_em.quantize(zt, e, m, rounding_mode=mode, grid=grid))
        for mode in rounding.MODES:
            for e, m in [(4, 3), (5, 2), (3, 2), (2, 3), (2, 1)]:
                out[f"float_em/ocp/{mode}/{e}/{m}"] = N(float_em.quantize(zt, e, m, rounding_mode=mode, grid="ocp"))
        # float64 inputs
        rng = np.random.default_rng(7)
        z64 = np.concatenate([z.astype(np.float64)[:4000],
                              rng.standard_normal(2000) * 2.0 ** rng.uniform(-140, 130, 2000),
                              (z.astype(np.float64)[:4000] * (1 + 2.0 ** -30))])
        out["corpus64"] = z64
        for grid, em in (("ieee", [(8, 7), (8, 23), (4, 4), (5, 10), (8, 12)]), ("ocp", [(4, 3), (2, 1)]),
                         ("qtorch", [(4, 3), (8, 7)])):
            for mode in rounding.MODES:
                for e, m in em:
                    out[f"float_em64/{grid}/{mode}/{e}/{m}"] = N(float_em.quantize(T(z64, torch.float64), e, m,
                                                                                   rounding_mode=mode, grid=grid))
        bits = z.view(np.uint32).astype(np.int64)
        bits = np.concatenate([bits, rng.integers(-2 ** 40, 2 ** 40, 2000)])
        keep = rng.integers(0, 23, bits.size)
        out["round_bits/bits"] = bits
        out["round_bits/keep"] = keep
        for mode in rounding.MODES:
            out[f"round_bits/{mode}"] = N(rounding.round_bits(torch.tensor(bits), torch.tensor(keep), mode))
            out[f"round_bits/{mode}/k7"] = N(rounding.round_bits(torch.tensor(bits), 7, mode))
        kk = np.concatenate([z, (rng.standard_normal(3000) * 40).astype(np.float32),
                             (np.arange(-40, 40) / 4).astype(np.float32)])
        out["round_int/in"] = kk
        for mode in rounding.MODES:
            out[f"round_int/{mode}"] = N(rounding.round_int(T(kk), mode))
            out[f"round_int64/{mode}"] = N(rounding.round_int(T(kk, torch.float64) * 1.5, mode))
        out["bf16"] = N(rounding.bf16(zt))
        for fmt in ("MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4"):
            for mode in ("nearest", "floor", "even"):
                out[f"microsoft/{fmt}/{mode}/sat"] = N(microsoft.quantize(zt, fmt, rounding_mode=mode))
                from mxq.microxcaling.elemwise import _quantize_elemwise
                from mxq.microxcaling.formats import ElemFormat
                from mxq.element_quant.formats import get
                out[f"microsoft/{fmt}/{mode}/nosat"] = N(_quantize_elemwise(
                    zt, ElemFormat.from_str(get(fmt).ocp), round=mode, saturate_normals=False, allow_denorm=True))
        amax = np.abs(z)
        at = T(amax)
        out["amax"] = amax
        for fl in (1e-38, 2.0 ** -23, 0.0, 1.0, 3e-39):
            out[f"scale/mxquant/{fl!r}"] = N(scale_factor.mxquant(at, fl))
        for emax in (8, 15, 4, 2):
            for sb in (8, 5):
                out[f"scale/ocp/{emax}/{sb}"] = N(scale_factor.ocp(at, emax, sb))
                out[f"scale/ocp_below_top/{emax}/{sb}"] = N(scale_factor.ocp_below_top(at, emax, sb))
        for fmt in ("MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4"):
            for mode in ("nearest", "floor", "even"):
                out[f"scale/ocp_no_clip/{fmt}/{mode}"] = N(scale_factor.ocp_no_clip(at, fmt, mode))
        # arith
        for m in (0, 1, 3, 7, 22, 23):
            out[f"truncate_significand/{m}"] = N(arith.truncate_significand(zt, m))
        for fe in (-16, -126, -150, 0):
            out[f"flush_product/{fe}"] = N(arith.flush_product(zt, fe))
        for lim, val in ((448.0, 448.0), (480.0, 480.0), (61440.0, 98304.0), (15.5, 30.0), (3.4e38, float("inf"))):
            out[f"saturate/{lim!r}/{val!r}"] = N(arith.saturate(zt, lim, val))
        ADD = [(4, 4), (4, 5), (4, 6), (4, 9), (4, 10), (3, 2), (5, 6), (7, 10), (6, 17), (8, 7), (8, 12), (8, 23),
               (2, 21), (3, 18)]
        for i, (e, m) in enumerate(ADD):
            a = grid_values(np, torch, float_em, e, m, 3000, 100 + i)
            b = grid_values(np, torch, float_em, e, m, 3000, 200 + i)
            # adversarial: near-cancellation and exact negatives, specials
            b[:300] = -a[:300]
            b[300:600] = a[300:600] * np.float32(1.0 + 2.0 ** -m)
            a[600:610] = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, np.inf, 0.0, -0.0, 1.0, -1.0], np.float32)
            b[600:610] = np.array([-np.inf, 1.0, 2.0, -0.0, 0.0, np.inf, 3.0, -2.0, np.nan, 0.0], np.float32)
            out[f"exact_add/{e}/{m}/a"] = a
            out[f"exact_add/{e}/{m}/b"] = b
            out[f"exact_add/{e}/{m}"] = N(arith.exact_add(T(a), T(b), e, m))
        for e, m, mode, grid in ((4, 4, "ties_away", "ieee"), (5, 6, "truncate", "ieee"), (4, 3, "rne", "ocp"),
                                 (4, 3, "ties_away", "qtorch"), (8, 7, "ties_away", "qtorch")):
            a = grid_values(np, torch, float_em, min(e, 8), m, 2000, 300)
            b = grid_values(np, torch, float_em, min(e, 8), m, 2000, 301)
            out[f"exact_add_g/{e}/{m}/{mode}/{grid}/a"] = a
            out[f"exact_add_g/{e}/{m}/{mode}/{grid}/b"] = b
            out[f"exact_add_g/{e}/{m}/{mode}/{grid}"] = N(arith.exact_add(T(a), T(b), e, m, mode, grid))
        np.savez_compressed(os.path.join(HERE, "elementwise.npz"), **out)
        print("elementwise.npz:", len(out), "arrays", flush=True)

    # --------------------------------------------------------------------------------- block quantizers
    if want("block"):
        out = {}
        rng = np.random.default_rng(2)
        R, Cc = 64, 128
        V = rng.standard_normal((R, Cc)) * 2.0 ** rng.uniform(-20, 20, (R, 1))
        V[rng.random((R, Cc)) < 0.01] = 0.0
        sub = rng.random((R, Cc)) < 0.001
        V[sub] = np.sign(rng.standard_normal(sub.sum())) * rng.uniform(2.0 ** -149, 2.0 ** -126, sub.sum())
        V = V.astype(np.float32)
        V[0:32, 5] = 0.0                                       # an all-zero block down a column
        V[3, 0:32] = 0.0                                       # and along a row
        V[32:64, 9] = (rng.uniform(-1, 1, 32) * 2.0 ** -140).astype(np.float32)   # subnormal-only block
        V[7, 40] = np.inf
        V[9, 70] = -np.inf
        V[11, 100] = np.nan
        V[50, 120] = np.float32(1.9999999)                     # near a binade top
        V[51, 121] = np.float32(2 ** 100 * (1 - 2 ** -24 * 10))
        out["V"] = V
        Vt = T(V)
        FMTS = ("MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4")
        for fam, q in (("mxquant", block.mxquant), ("mxgemmini", block.mxgemmini), ("ocp", block.ocp)):
            for fmt in FMTS:
                for axis in (0, 1):
                    P, X = q.quantize(Vt, fmt, axis=axis)
                    out[f"{fam}/{fmt}/{axis}/P"], out[f"{fam}/{fmt}/{axis}/X"] = N(P), N(X)
        for fmt in ("MXFP8_E4M3", "MXFP6_E2M3"):
            for mode in ("rne", "truncate"):
                for fl in (2.0 ** -23, 1e-38):
                    P, X = block.mxgemmini.quantize(Vt, fmt, axis=0, rounding_mode=mode, scale_floor=fl)
                    out[f"mxgemmini_k/{fmt}/{mode}/{fl!r}/P"], out[f"mxgemmini_k/{fmt}/{mode}/{fl!r}/X"] = N(P), N(X)
        P, X = block.mxgemmini.quantize(Vt, "MXFP4", axis=0, rounding_mode="rne", via=(3, 1))
        out["mxgemmini_via/P"], out["mxgemmini_via/X"] = N(P), N(X)
        for fmt in ("MXFP8_E4M3", "MXFP6_E3M2"):
            for pl in ("below_top", "no_clip"):
                for mode in ("nearest", "even"):
                    P, X = block.ocp.quantize(Vt, fmt, axis=1, rounding_mode=mode, placement=pl)
                    out[f"ocp_p/{fmt}/{pl}/{mode}/P"], out[f"ocp_p/{fmt}/{pl}/{mode}/X"] = N(P), N(X)
            P, X = block.ocp.quantize(Vt, fmt, axis=0, rounding_mode="floor", scale_bits=5)
            out[f"ocp_sb/{fmt}/P"], out[f"ocp_sb/{fmt}/X"] = N(P), N(X)
        P, X = block.mxgemmini.quantize(Vt, "FP32", axis=0)
        out["fp32/P"], out["fp32/X"] = N(P), N(X)
        # odd shapes and block sizes
        V3 = (rng.standard_normal((4, 37, 10)) * 2.0 ** rng.uniform(-5, 5, (4, 1, 10))).astype(np.float32)
        out["V3"] = V3
        for fam, q in (("mxquant", block.mxquant), ("mxgemmini", block.mxgemmini), ("ocp", block.ocp)):
            for axis in (0, 1, 2, -1):
                P, X = q.quantize(T(V3), "MXFP8_E4M3", axis=axis)
                out[f"odd/{fam}/{axis}/P"], out[f"odd/{fam}/{axis}/X"] = N(P), N(X)
            for bs in (16, 7):
                P, X = q.quantize(T(V3), "MXFP6_E2M3", axis=1, block_size=bs)
                out[f"bs/{fam}/{bs}/P"], out[f"bs/{fam}/{bs}/X"] = N(P), N(X)
        np.savez_compressed(os.path.join(HERE, "block.npz"), **out)
        print("block.npz:", len(out), "arrays", flush=True)

    # ------------------------------------------------------------------------------------------- reducers
    if want("reducers"):
        out = {}
        # config 1 (the PR1 reference workload), full size: inputs are regenerated from the seed by the tests
        g = torch.Generator().manual_seed(0)
        x = torch.randn(256, 512, generator=g)
        W = torch.randn(512, 512, generator=g)
        P_A, X_A = block.mxgemmini.quantize(x.t(), "MXFP8_E4M3", axis=0)
        P_B, X_B = block.mxgemmini.quantize(W.t(), "MXFP8_E4M3", axis=0)
        t0 = time.time()
        Y = matmul.systolic(P_A, X_A, P_B, X_B, matmul.MXGEMMINI(), schedule.HW_FINAL)
        print(f"config 1 systolic: {time.time() - t0:.1f}s", flush=True)
        out["config1/x_sum"] = np.float64(x.double().sum())
        out["config1/W_sum"] = np.float64(W.double().sum())
        out["config1/Y"] = N(Y)
        out["config1/P_A"], out["config1/X_A"], out["config1/P_B"], out["config1/X_B"] = N(P_A), N(X_A), N(P_B), N(X_B)

        rng = np.random.default_rng(3)

        def operands(K, M, Nn, fmt, seed, special=False, scale=1.0, rounding_mode="ties_away", floor=1e-38):
            r = np.random.default_rng(seed)
            A = (r.standard_normal((K, M)) * scale * 2.0 ** r.uniform(-6, 6, (1, M))).astype(np.float32)
            B = (r.standard_normal((K, Nn)) * scale * 2.0 ** r.uniform(-6, 6, (1, Nn))).astype(np.float32)
            A[r.random((K, M)) < 0.05] = 0.0
            pa, xa = block.mxgemmini.quantize(T(A), fmt, axis=0, rounding_mode=rounding_mode, scale_floor=floor)
            pb, xb = block.mxgemmini.quantize(T(B), fmt, axis=0, rounding_mode=rounding_mode, scale_floor=floor)
            pa, xa, pb, xb = N(pa), N(xa), N(pb), N(xb)
            if special:
                pa[1, 2] = np.inf
                pb[5, 3] = np.nan
                pa[7, 4] = -np.inf
                pb[7, 4] = 0.0
                pa[9, 6] = 300.0
                pb[9, 6] = 3.0
                pa[10, 7] = 2.0 ** -20
                pb[10, 7] = 2.0 ** -3
                xa[0, 8] = np.float32(2.0 ** 120)
                xb[0, 8] = np.float32(2.0 ** 20)
                xa[0, 9] = np.float32(2.0 ** -140)
            return pa, xa, pb, xb

        cases = []
        HW = list(schedule.HW_FINAL)
        for K in (96, 80, 70):
            cases.append((f"sys/mxg/hw/K{K}", "systolic", ("mxg", 4, 3, -16), HW, 16, dict(K=K)))
        cases += [
            ("sys/mxg/hw/special", "systolic", ("mxg", 4, 3, -16), HW, 16, dict(K=96, special=True)),
            ("sys/mxg/hw/e2m3", "systolic", ("mxg", 4, 3, -16), HW, 16, dict(K=96, fmt="MXFP6_E2M3")),
            ("sys/mxg/hw/rne_hwfloor", "systolic", ("mxg", 4, 3, -16), HW, 16,
             dict(K=96, rounding_mode="rne", floor=2.0 ** -23)),
            ("sys/mxg/bf16", "systolic", ("mxg", 4, 3, -16), [(8, 7)] * 16, 16, dict(K=96)),
            ("sys/mxg/e5m6", "systolic", ("mxg", 4, 3, -16), [(5, 6)] * 16, 16, dict(K=96)),
            ("sys/mxg/desc", "systolic", ("mxg", 4, 3, -16), [(4, 6)] * 4 + [(4, 4)] * 4 + [(3, 3)] * 4 + [(8, 7)] * 4,
             16, dict(K=96, special=True)),
            ("sys/mxg/f32lanes", "systolic", ("mxg", 4, 3, -16), [(8, 23)] * 16, 16, dict(K=96)),
            ("sys/mxg/e7m10", "systolic", ("mxg", 4, 3, -16), [(7, 10)] * 16, 16, dict(K=96)),
            ("sys/mxg/p44nofloor", "systolic", ("mxg", 4, 4, None), HW, 16, dict(K=96)),
            ("sys/mxg/p52", "systolic", ("mxg", 5, 2, -16), HW, 16, dict(K=96, special=True)),
            ("sys/mxg/p87", "systolic", ("mxg", 8, 7, -16), [(8, 7)] * 16, 16, dict(K=96, special=True)),
            ("sys/mxg/size8", "systolic", ("mxg", 4, 3, -16), HW[:7] + [(8, 7)], 8, dict(K=96)),
            ("sys/mxg/size32", "systolic", ("mxg", 4, 3, -16), HW + HW, 32, dict(K=70)),
            ("sys/mxq/43", "systolic", ("mxq", 4, 3), HW, 16, dict(K=96)),
            ("sys/mxq/43/special", "systolic", ("mxq", 4, 3), HW, 16, dict(K=96, special=True)),
            ("sys/mxq/52", "systolic", ("mxq", 5, 2), [(5, 10)] * 16, 16, dict(K=80)),
            ("sys/mxq/87", "systolic", ("mxq", 8, 7), [(8, 23)] * 16, 16, dict(K=96)),
            ("add/mxg/ladder", "adder", ("mxg", 4, 3, -16), [(4, 4), (4, 5), (4, 6), (8, 7)], 16, dict(K=96)),
            ("add/mxg/ladder/K70", "adder", ("mxg", 4, 3, -16), [(4, 4), (4, 5), (4, 6), (8, 7)], 16,
             dict(K=70, special=True)),
            ("add/mxg/size8", "adder", ("mxg", 4, 3, -16), [(8, 7)] * 3, 8, dict(K=96)),
            ("add/mxq", "adder", ("mxq", 4, 3), [(4, 4), (4, 5), (4, 6), (8, 7)], 16, dict(K=96)),
            ("anc/mxg/default", "anchor", ("mxg", 4, 3, -16), None, 16, dict(K=96)),
            ("anc/mxg/default/K70", "anchor", ("mxg", 4, 3, -16), None, 16, dict(K=70, special=True)),
            ("anc/mxg/w8", "anchor", ("mxg", 4, 3, -16), None, 16, dict(K=96, width=8)),
            ("anc/mxg/w4rne", "anchor", ("mxg", 4, 3, -16), [(4, 6), (4, 6), (8, 7), (8, 7)], 16,
             dict(K=96, width=4, drop="rne", headroom=6)),
            ("anc/mxg/bits", "anchor", ("mxg", 4, 3, -16), None, 16, dict(K=96, bits=[21, 20, 18, 16, 14, 12], emin=-10)),
            ("anc/mxq", "anchor", ("mxq", 4, 3), [(4, 6)], 16, dict(K=96)),
            ("fp64", "fp64", None, None, 16, dict(K=96)),
        ]
        M, Nn = 24, 20
        for i, (name, red, ar, sched, size, kw) in enumerate(cases):
            kw = dict(kw)
            K = kw.pop("K")
            fmt = kw.pop("fmt", "MXFP8_E4M3")
            special = kw.pop("special", False)
            rm = kw.pop("rounding_mode", "ties_away")
            fl = kw.pop("floor", 1e-38)
            pa, xa, pb, xb = operands(K, M, Nn, fmt, 1000 + i, special, rounding_mode=rm, floor=fl)
            for k, v in (("P_A", pa), ("X_A", xa), ("P_B", pb), ("X_B", xb)):
                out[f"{name}/{k}"] = v
            if ar is None:
                A = None
            elif ar[0] == "mxg":
                A = matmul.MXGEMMINI(ar[1], ar[2], ar[3])
            else:
                A = matmul.MXQUANT(ar[1], ar[2])
            args = (T(pa), T(xa), T(pb), T(xb))
            if red == "systolic":
                Yr = matmul.systolic(*args, A, sched, size=size)
            elif red == "adder":
                Yr = matmul.adder_tree(*args, A, sched, size=size)
            elif red == "anchor":
                Yr = matmul.anchor_tree(*args, A, sched, size=size, **kw)
            else:
                Yr = fp64_accum(*args)
            out[f"{name}/Y"] = N(Yr)
        meta = {name: dict(reducer=red, arith=ar, schedule=sched, size=size,
                           kw={k: v for k, v in kw.items() if k not in ("K", "fmt", "special", "rounding_mode", "floor")})
                for name, red, ar, sched, size, kw in cases}
        out["meta"] = np.array(json.dumps(meta))
        np.savez_compressed(os.path.join(HERE, "reducers.npz"), **out)
        print("reducers.npz:", len(out), "arrays", flush=True)

    # ------------------------------------------------------------------------------------------------ LUT
    if want("lut"):
        from mxq.lut import formats as lf
        out = {}
        rng = np.random.default_rng(4)
        K, n = 128, 40
        V = (rng.standard_normal((K, n)) * 2.0 ** rng.uniform(-8, 8, (1, n))).astype(np.float32)
        V[:, 6:8] = np.round(V[:, 6:8])                         # few distinct codes in one group
        out["V"] = V
        for fmt in lut.FORMATS:
            vals = lf._tables(lf._format(fmt).name)
            out[f"tables/{fmt}/vals"], out[f"tables/{fmt}/fx"], out[f"tables/{fmt}/safe"] = (N(vals[0]), N(vals[1]),
                                                                                             N(vals[2]))
            for G in (0, 1, 3):
                for axis in (0, 1):
                    P_l, X_l = block.lut.quantize(T(V), fmt, axis=axis, block_size=32, rounding_mode="rne",
                                                  scale_floor=2.0 ** -23, group=G, max_iters=50)
                    out[f"blut/{fmt}/{G}/{axis}/P"], out[f"blut/{fmt}/{G}/{axis}/X"] = N(P_l), N(X_l)
                P, _ = block.mxgemmini.quantize(T(V), fmt, axis=0, rounding_mode="rne", scale_floor=2.0 ** -23)
                Tt = lut.tables(P, fmt, group=G, max_iters=50)
                I = lut.pick(P, Tt, group=G)
                out[f"lut/{fmt}/{G}/P"], out[f"lut/{fmt}/{G}/T"], out[f"lut/{fmt}/{G}/I"] = N(P), N(Tt), N(I)
                out[f"lut/{fmt}/{G}/lookup"] = N(lut.lookup(I, Tt, group=G))
                Tt5 = lut.tables(P, fmt, group=G, max_iters=2)
                out[f"lut/{fmt}/{G}/T_it2"] = N(Tt5)
                if n % (1 << G) == 0:
                    codes = lut.encode(P, fmt)
                    out[f"lut/{fmt}/{G}/codes"] = N(codes)
                    out[f"lut/{fmt}/{G}/finder"] = N(lut.finder(codes, Tt, fmt, group=G))
                    out[f"lut/{fmt}/{G}/Tcodes"] = N(lut.encode(Tt, fmt))
                    if G == 1:                                  # negative codes index from the end, as torch does
                        nc = lf._tables(lf._format(fmt).name)[0].numel()
                        neg = codes.clone()
                        neg[::3] -= nc
                        out[f"lut/{fmt}/codes_neg"] = N(neg)
                        out[f"lut/{fmt}/decode_neg"] = N(lut.decode(neg, fmt))
                        out[f"lut/{fmt}/finder_neg"] = N(lut.finder(neg, Tt, fmt, group=G))
        np.savez_compressed(os.path.join(HERE, "lut.npz"), **out)
        print("lut.npz:", len(out), "arrays", flush=True)

    # ------------------------------------------------------------------------------------------- model
    if want("model"):
        from functools import partial
        from mxq import Scheme
        from mxq.nn import patch
        from transformers import LlamaConfig, LlamaForCausalLM
        out = {}
        cfg = LlamaConfig(hidden_size=128, intermediate_size=352, num_hidden_layers=2, num_attention_heads=4,
                          num_key_value_heads=4, head_dim=32, vocab_size=256, max_position_embeddings=128,
                          initializer_range=0.02)
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg).float().eval()
        ids = torch.randint(0, 256, (2, 40), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            out["logits_plain"] = N(model(ids).logits)
        q = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
        s = Scheme("hw_fp8", a=q, b=q, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(), schedule=schedule.HW_FINAL))
        patch(model, [("lm_head", None), ("model.layers.*.self_attn", (s, s)), (torch.nn.Linear, s)])
        captured = {}

        def hook(name):
            def f(mod, inp, outp):
                captured[name + "/x"] = N(inp[0])
                captured[name + "/y"] = N(outp)
            return f
        for name, mod in model.named_modules():
            if type(mod).__name__ == "MXLinear":
                mod.register_forward_hook(hook(name))
        with torch.no_grad():
            out["logits"] = N(model(ids).logits)
        out.update(captured)
        out["ids"] = N(ids)
        np.savez_compressed(os.path.join(HERE, "model.npz"), **out)
        print("model.npz:", len(out), "arrays", flush=True)

    # ------------------------------------------------------------------------------------------------- nn
    if want("nn"):
        from functools import partial
        from mxq import Scheme
        from mxq.nn import MXLinear, attend
        out = {}
        q = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
        hw = Scheme("hw", a=q, b=q, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(), schedule=schedule.HW_FINAL))
        g = torch.Generator().manual_seed(5)
        lin = torch.nn.Linear(96, 40, bias=True)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(40, 96, generator=g) * 0.1)
            lin.bias.copy_(torch.randn(40, generator=g))
        xin = torch.randn(3, 11, 96, generator=g)
        out["linear/W"], out["linear/b"], out["linear/x"] = N(lin.weight), N(lin.bias), N(xin)
        out["linear/y"] = N(MXLinear(lin, hw)(xin))
        out["linear/y_chunk5"] = N(MXLinear(lin, hw, chunk=5)(xin))
        qa, ka, va = (torch.randn(2, 4, 9, 32, generator=g), torch.randn(2, 2, 12, 32, generator=g),
                      torch.randn(2, 2, 12, 32, generator=g))
        mask = torch.zeros(2, 1, 9, 12)
        mask[1, :, :, :3] = torch.finfo(torch.float32).min
        causal = torch.triu(torch.full((9, 12), torch.finfo(torch.float32).min), diagonal=4)
        mask[0, 0] = causal
        out["attend/q"], out["attend/k"], out["attend/v"], out["attend/mask"] = N(qa), N(ka), N(va), N(mask)
        out["attend/o"] = N(attend(qa, ka, va, mask, 32 ** -0.5, hw, hw))
        out["attend/o_nomask"] = N(attend(qa, ka, va, None, 32 ** -0.5, hw, hw))
        out["attend/o_chunk4"] = N(attend(qa, ka, va, mask, 32 ** -0.5, hw, hw, chunk=4))
        A = torch.randn(96, 7, generator=g)
        B = torch.randn(96, 5, generator=g)
        out["scheme/A"], out["scheme/B"], out["scheme/Y"] = N(A), N(B), N(hw.matmul(A, B))
        np.savez_compressed(os.path.join(HERE, "nn.npz"), **out)
        print("nn.npz:", len(out), "arrays", flush=True)


    # ------------------------------------------------------------------------- the rest of the public API
    if want("api"):
        api(np, torch, T, N)


def api(np, torch, T, N):
    """api.npz: the rounding modules' bits / integer forms, block.compose with scale_factor / element_quant
    callables and the blocking helpers, schedule.load / fixed (results and error messages), the vector ops and
    vector="bf16" through patch, attend on decode / GQA / multi-chunk causal shapes, patch's dry-run table and
    errors, and mxq.nn.torchao.MXQConfig (imported with a stand-in for the absent torchao: only its base class and
    handler registry are touched)."""
    import tempfile
    import types
    from functools import partial
    from mxq import block, matmul, rounding, scale_factor, schedule
    from mxq.block import _driver
    from mxq.element_quant import float_em, microsoft
    out, msgs = {}, {}

    # rounding.{rne,ties_away,truncate}.bits / integer
    rng = np.random.default_rng(21)
    bits = np.concatenate([hard_corpus(np, 500).view(np.uint32).astype(np.int64),
                           np.array([0xFFFFFFFF, 0xFFFFFFF0, 0x7FFFFFFF, 0xFFFF8000, 0xFFFFFFFF << 4, -1, -2 ** 40,
                                     2 ** 40 + 12345, 0x80000000, 0x7F7FFFFF], np.int64),
                           rng.integers(-2 ** 45, 2 ** 45, 500)])
    out["rbits/bits"] = bits
    keep = rng.integers(0, 23, bits.size)
    out["rbits/keep"] = keep
    bt = torch.tensor(bits)
    kk = np.concatenate([(rng.standard_normal(400) * 40).astype(np.float32), np.arange(-20, 20) / 4])
    out["rint/in"] = kk.astype(np.float32)
    for name, mod in (("rne", rounding.rne), ("ties_away", rounding.ties_away), ("truncate", rounding.truncate)):
        for k in (0, 3, 7, 10, 22):
            drop = 23 - k
            out[f"rbits/{name}/{k}"] = N(mod.bits(bt, drop, (1 << drop) - 1, 1 << (drop - 1)))
        d, m, h = rounding._drop(bt, torch.tensor(keep))
        out[f"rbits/{name}/tensor"] = N(mod.bits(bt, d, m, h))
        out[f"rint/{name}/f32"] = N(mod.integer(T(kk)))
        out[f"rint/{name}/f64"] = N(mod.integer(T(kk, torch.float64) * 1.5))

    # block.compose with the reference's own steps, and the blocking helpers
    V3 = (rng.standard_normal((3, 45, 6)) * 2.0 ** rng.uniform(-12, 12, (3, 1, 6))).astype(np.float32)
    V3[0, :32, 0] = 0.0
    V3[1, 5, 2] = np.float32(2.0 ** -140)
    out["compose/V"] = V3
    steps = {
        "mxquant_hwfloor": (partial(scale_factor.mxquant, floor=2.0 ** -23),
                            partial(float_em.quantize, e=4, m=3, rounding_mode="ties_away", grid="qtorch")),
        "ocp_microsoft": (partial(scale_factor.ocp, emax=8), partial(microsoft.quantize, fmt="MXFP8_E4M3")),
        "mxquant_ocp_rne": (scale_factor.mxquant, partial(float_em.quantize, e=3, m=2, rounding_mode="rne",
                                                           grid="ocp")),
        "below_top": (partial(scale_factor.ocp_below_top, emax=4),
                      partial(microsoft.quantize, fmt="MXFP6_E3M2", rounding_mode="nearest")),
        "no_clip": (partial(scale_factor.ocp_no_clip, fmt="MXFP6_E2M3"), partial(microsoft.quantize, fmt="MXFP6_E2M3")),
        "ieee_truncate": (partial(scale_factor.ocp, emax=15, scale_bits=5),
                          partial(float_em.quantize, e=5, m=2, rounding_mode="truncate", grid="ieee")),
        "no_scale": (None, partial(float_em.quantize, e=4, m=3, rounding_mode="rne", grid="ocp")),
        "no_elem": (scale_factor.mxquant, None),
        "neither": (None, None),
    }
    for name, (sc, el) in steps.items():
        for axis, bs in ((0, 32), (1, 32), (1, 16), (2, 4), (-1, 3), (1, 7)):
            P, X = block.compose(T(V3), scale=sc, elem=el, axis=axis, block_size=bs)
            out[f"compose/{name}/{axis}/{bs}/P"], out[f"compose/{name}/{axis}/{bs}/X"] = N(P), N(X)
    for axis, bs in ((0, 32), (1, 16), (1, 7), (2, 4)):
        b = _driver.to_blocks(T(V3), axis, bs)
        out[f"blocks/{axis}/{bs}/data"] = N(b.data)
        out[f"blocks/{axis}/{bs}/codes"] = N(_driver.codes_from_blocks(b.data * 2 + 1, b))
        out[f"blocks/{axis}/{bs}/scales"] = N(_driver.scales_from_blocks(b.data.abs().amax(-1, keepdim=True), b))
        Xb = _driver.scales_from_blocks(b.data.abs().amax(-1, keepdim=True), b)
        out[f"blocks/{axis}/{bs}/dequantize"] = N(block.dequantize(T(V3), Xb, axis=axis, block_size=bs))

    # schedule.load / fixed
    hw = "\n".join(f"{i},{e},{m}" for i, (e, m) in enumerate(schedule.HW_FINAL))
    csvs = {
        "header3": "position,e,m\n" + hw + "\n",
        "plain3": hw + "\n",
        "four": "pos,B,e,m\n" + "\n".join(f"{15 - i}, 32 ,{e},{m}" for i, (e, m) in enumerate(schedule.HW_FINAL[::-1])),
        "skips": "# lanes\n" + "\n".join(f"{i},{e},{m}\n{i},x" for i, (e, m) in enumerate(schedule.HW_FINAL)) + "\n,,\n",
        "rows8": "\n".join(f"{i},4,{3 + i}" for i in range(8)),
        "twice": hw + "\n3,4,4\n",
        "outside": hw + "\n16,4,4\n",
        "negative": hw + "\n-1,4,4\n",
        "missing": "\n".join(f"{i},4,4" for i in range(16) if i not in (2, 11)),
        "empty": "",
        "header_only": "position,e,m\n",
    }
    msgs["schedule/csv"] = csvs
    with tempfile.TemporaryDirectory() as d:
        for name, text in csvs.items():
            path = os.path.join(d, name + ".csv")
            with open(path, "w") as f:
                f.write(text)
            rows = 8 if name == "rows8" else 16
            try:
                msgs[f"schedule/{name}"] = {"ok": [list(x) for x in schedule.load(path, rows=rows)], "rows": rows}
            except ValueError as e:
                msgs[f"schedule/{name}"] = {"error": str(e).replace(path, "<path>"), "rows": rows}
    msgs["schedule/fixed"] = [list(x) for x in schedule.fixed(5, 6, rows=4)]

    # the vector ops, and attend on more shapes
    from mxq import Scheme
    from mxq.nn import attend, _vector
    S = (rng.standard_normal((6, 40)) * 4).astype(np.float32)
    S[2, 30:] = np.finfo(np.float32).min
    out["vector/S"] = S
    out["vector/softmax_bf16"] = N(_vector.softmax(T(S), "bf16"))
    xr = (rng.standard_normal((5, 64)) * 3).astype(np.float32)
    wr = (1 + rng.standard_normal(64) * 0.1).astype(np.float32)
    out["vector/x"], out["vector/w"] = xr, wr
    out["vector/rmsnorm_bf16"] = N(_vector.rmsnorm(T(xr), T(wr), 1e-6, "bf16"))
    out["vector/rmsnorm_none"] = N(_vector.rmsnorm(T(xr), T(wr), 1e-6, None))
    q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    hw_s = Scheme("hw", a=q8, b=q8, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(), schedule=schedule.HW_FINAL))
    g = torch.Generator().manual_seed(22)
    fmin = torch.finfo(torch.float32).min
    shapes = {
        "decode": (2, 4, 1, 23, 2, None),                    # B, H, Tq, Tk, Hkv, chunk
        "gqa4": (1, 8, 12, 12, 2, None),
        "causal_chunks": (2, 4, 64, 64, 2, 16),
        "padded_chunks": (2, 2, 40, 40, 1, 8),
    }
    for name, (B, H, Tq, Tk, Hkv, ch) in shapes.items():
        qa = torch.randn(B, H, Tq, 32, generator=g)
        ka = torch.randn(B, Hkv, Tk, 32, generator=g)
        va = torch.randn(B, Hkv, Tk, 32, generator=g)
        mask = torch.triu(torch.full((Tq, Tk), fmin), diagonal=Tk - Tq + 1)[None, None].repeat(B, 1, 1, 1)
        if name == "padded_chunks":
            mask[1, :, :, :9] = fmin                         # left padding of batch row 1
        for k_, t in (("q", qa), ("k", ka), ("v", va), ("mask", mask)):
            out[f"attend/{name}/{k_}"] = N(t)
        out[f"attend/{name}/o"] = N(attend(qa, ka, va, mask, 32 ** -0.5, hw_s, hw_s, chunk=ch))
        out[f"attend/{name}/o_bf16"] = N(attend(qa, ka, va, mask, 32 ** -0.5, hw_s, hw_s, chunk=ch, vector="bf16"))

    # vector="bf16" through patch, and patch's dry-run table and errors
    from mxq.nn import patch, is_attention
    from transformers import LlamaConfig, LlamaForCausalLM
    import contextlib
    import io
    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, vocab_size=128, max_position_embeddings=64,
                      initializer_range=0.02)
    ids = torch.randint(0, 128, (2, 24), generator=torch.Generator().manual_seed(23))
    out["model/ids"] = N(ids)
    settings = {"bf16": ([("lm_head", None), ("model.layers.*.self_attn", (hw_s, hw_s)), (torch.nn.Linear, hw_s)],
                         "bf16"),
                "rmsnorm": ([("lm_head", None), (torch.nn.Linear, hw_s)], {"rmsnorm": "bf16"}),
                "softmax_exact": ([("lm_head", None), (is_attention, None), (torch.nn.Linear, hw_s)],
                                  {"softmax": "bf16"})}
    for name, (rules, vec) in settings.items():
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg).float().eval()
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            patch(model, rules, dry_run=True, vector=vec)
        msgs[f"patch/{name}/dry_run"] = buf.getvalue()
        handle = patch(model, rules, vector=vec)
        with torch.no_grad():
            out[f"model/{name}/logits"] = N(model(ids).logits)
        handle.revert()
        with torch.no_grad():
            out[f"model/{name}/logits_reverted"] = N(model(ids).logits)

    class Twice(torch.nn.Module):                            # one Linear held in two places
        def __init__(self):
            super().__init__()
            self.a = torch.nn.Linear(32, 16)
            self.b = self.a
            self.c = torch.nn.Linear(16, 8)
            self.att = torch.nn.Module()                     # an attention module: it holds q_proj and k_proj
            self.att.q_proj = torch.nn.Linear(32, 32)
            self.att.k_proj = torch.nn.Linear(32, 32)
    errors = {
        "bad_rule": lambda m: patch(m, [("a", "fp8")]),
        "no_linear": lambda m: patch(m, [("nothing.*", hw_s), (torch.nn.Linear, None)]),
        "hidden": lambda m: patch(m, [(torch.nn.Linear, None), ("c", hw_s)]),
        "two_rules": lambda m: patch(m, [("a", hw_s), ("b", None), (torch.nn.Linear, None)]),
        "no_core": lambda m: patch(m, [("x", (hw_s, hw_s))]),
        "softmax_no_attention": lambda m: patch(m, [], vector="bf16"),
        "vector_spelling": lambda m: patch(m, [], vector={"softmax": "fp16"}),
    }
    class Shared(torch.nn.Module):                           # a whole subtree held twice: one attribute, two names
        def __init__(self):
            super().__init__()
            self.x = Twice()
            self.y = self.x
    errors["same_site"] = lambda m: patch(Shared(), [("x.c", hw_s), ("y.c", None), (torch.nn.Linear, None)])
    errors["same_core"] = lambda m: patch(Shared(), [("x.att", (hw_s, hw_s)), (torch.nn.Linear, None)])
    for name, fn in errors.items():
        try:
            fn(Twice())
            msgs[f"patch_error/{name}"] = None
        except ValueError as e:
            msgs[f"patch_error/{name}"] = str(e)
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        patch(Twice(), [("c", None), (torch.nn.Linear, hw_s)], dry_run=True)
    msgs["patch/twice/dry_run"] = buf.getvalue()
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        patch(Shared(), [("*.c", None), ("*.att", (hw_s, hw_s)), (is_attention, None), (torch.nn.Linear, hw_s)],
              dry_run=True, vector={"rmsnorm": None, "softmax": "bf16"})
    msgs["patch/shared/dry_run"] = buf.getvalue()

    # mxq.nn.torchao.MXQConfig, with a stand-in for torchao's two names (base class, handler registry)
    stub_core = types.ModuleType("torchao.core.config")

    class AOBaseConfig:
        pass
    stub_core.AOBaseConfig = AOBaseConfig
    stub_tm = types.ModuleType("torchao.quantization.transform_module")
    stub_tm.register_quantize_module_handler = lambda cls: (lambda fn: fn)
    for mname, mod in (("torchao", types.ModuleType("torchao")), ("torchao.core", types.ModuleType("torchao.core")),
                       ("torchao.core.config", stub_core),
                       ("torchao.quantization", types.ModuleType("torchao.quantization")),
                       ("torchao.quantization.transform_module", stub_tm)):
        sys.modules[mname] = mod
    from mxq.nn import torchao as mt
    from mxq.nn import MXLinear
    lin = torch.nn.Linear(64, 24)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(24, 64, generator=g) * 0.2)
        lin.bias.copy_(torch.randn(24, generator=g))
    x = torch.randn(2, 8, 64, generator=g)
    out["torchao/W"], out["torchao/b"], out["torchao/x"] = N(lin.weight), N(lin.bias), N(x)
    configs = {
        "default": {},
        "e2m3_truncate": {"fmt": "MXFP6_E2M3", "rounding_mode": "truncate", "scale_floor": 1e-38},
        "prod44_nofloor": {"prod": (4, 4), "prod_floor": None, "ladder": [[8, 7]] * 16},
        "exact": {"reduce": "exact"},
        "lut": {"fmt": "MXFP6_E3M2", "lut": {"group": 1, "max_iters": 5}},
        "size8": {"size": 8, "ladder": [[4, 6]] * 8, "block_size": 32, "chunk": 3},
        "via": {"fmt": "MXFP4", "via": [3, 1]},
    }
    for name, kw in configs.items():
        c = mt.MXQConfig(**kw)
        msgs[f"torchao/{name}/dict"] = c.to_dict()
        s = c.scheme("cpu")
        msgs[f"torchao/{name}/scheme"] = {"name": s.name, "rows": s.rows, "block_size": s.block_size}
        out[f"torchao/{name}/y"] = N(MXLinear(lin, s, chunk=c.chunk)(x))
    bad = {
        "fp32": {"fmt": "FP32"}, "reduce": {"reduce": "fast"}, "prod": {"prod": [4]},
        "ladder_len": {"ladder": [[4, 4]] * 15}, "prod_floor": {"prod_floor": 1.5},
        "block": {"block_size": 24}, "compiled": {"compiled": 1}, "chunk": {"chunk": 0},
        "lut_keys": {"fmt": "MXFP6_E3M2", "lut": {"group": 1}}, "lut_fmt": {"fmt": "MXFP4", "lut": {"group": 1, "max_iters": 2}},
        "lut_via": {"fmt": "MXFP6_E3M2", "via": [3, 1], "lut": {"group": 1, "max_iters": 2}},
        "ladder_entry": {"ladder": [[4, 4]] * 15 + [[4, 0]]}, "from_dict_type": None,
    }
    for name, kw in bad.items():
        try:
            if kw is None:
                mt.MXQConfig.from_dict({"_type": "Other", "_data": {}})
            else:
                mt.MXQConfig(**kw)
            msgs[f"torchao_error/{name}"] = None
        except ValueError as e:
            msgs[f"torchao_error/{name}"] = str(e)
    rt = mt.MXQConfig.from_dict({"_type": "MXQConfig", "_data": mt.MXQConfig(fmt="MXFP8_E5M2").to_dict()})
    msgs["torchao/roundtrip"] = rt.to_dict()
    out["msgs"] = np.array(json.dumps(msgs))
    np.savez_compressed(os.path.join(HERE, "api.npz"), **out)
    print("api.npz:", len(out), "arrays", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MXQ_REFERENCE"),
                    help="the reference checkout to import (default: $MXQ_REFERENCE)")
    ap.add_argument("--only", nargs="*", default=[])
    ap.add_argument("--child", action="store_true")
    a = ap.parse_args()
    if not a.child and not a.reference:
        ap.error("give the reference checkout with --reference or $MXQ_REFERENCE")
    if a.child:
        child(set(a.only))
        return
    env = dict(os.environ, PYTHONPATH=a.reference, PYTHONDONTWRITEBYTECODE="1", MXQ_REFERENCE=a.reference)
    subprocess.run([sys.executable, "-B", os.path.abspath(__file__), "--child", "--only", *a.only], env=env,
                   cwd="/", check=True)


if __name__ == "__main__":
    main()
