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
