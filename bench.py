"""Benchmark of the mxq B200 hot path (the driver's bench contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

Headline ("quantize GB/s"): the block-quantizer sweep. A step quantizes one float32
8192 x 8192 matrix -- N(0,1) x 2^U[-20,20] per row, 1% exact zeros, 0.1% float32-subnormal values -- with each of
block.mxquant / block.mxgemmini / block.ocp, each of the five MX formats, along axis 0 and axis 1: 30 fused kernel
launches. Throughput counts the algorithmic bytes of the reference's contract, 8.125 B per element (read V, write
P, write X once per 32 elements). Every rank quantizes its own row shard (weak scaling, no collective).

Beside it, in the same JSON line, `systolic`: config 3's 4096^3 MXFP8_E4M3 systolic GEMM (MXGEMMINI / HW_FINAL,
operands quantized by block.mxgemmini) in emulated GMAC/s, each rank reducing its own 4096-column panel of B;
`reducers`: config 3's reducers (systolic MXGEMMINI and MXQUANT(4,3), adder tree, anchor tree) timed alone.

`e2e` runs the same sweep through the public API with a pinned host V: every call streams V through the device in
chunks and returns host P and X (copies in, kernels and copies out overlapped on three streams), all inside the
timed region. `cpu_baseline` times the CPU oracle (oracle/, a C restatement of the reference algorithm; the
reference itself is Python and does not travel) on the same matrix, swept twice (about 10 s on 16 cores).
`--impl reference` is the reference arm: the oracle on all host cores, rank 0 only, same metric and unit.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "microscaling-quant_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

FAMILIES = ("mxquant", "mxgemmini", "ocp")
FORMATS = ("MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4")
ROWS, COLS = 8192, 8192
BYTES_PER_ELEM = 8.125
GEMM = 4096
METRIC = "bit-exact MX block-quantize GB/s (config 2 sweep: 3 quantizers x 5 formats x 2 axes)"
HW_FINAL = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]


def peaks():
    """Measured peaks (MEASURED_PEAKS.json, written by the driver), else the pool's fallback figures."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def synthetic(rows, cols, seed, device=None):
    """config 2's matrix, generated on the device (torch) or the host (numpy) from a seed."""
    import torch
    g = torch.Generator(device=device or "cpu").manual_seed(seed)
    V = torch.randn(rows, cols, generator=g, device=device) * torch.exp2(
        torch.rand(rows, 1, generator=g, device=device) * 40 - 20)
    zero = torch.rand(rows, cols, generator=g, device=device) < 0.01
    V[zero] = 0.0
    sub = torch.rand(rows, cols, generator=g, device=device) < 0.001
    mag = (torch.rand(rows, cols, generator=g, device=device) * (2.0 ** -126 - 2.0 ** -149) + 2.0 ** -149)
    V[sub] = (torch.sign(V) * mag)[sub]
    return V.contiguous()


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=lambda: self.lines.extend(self.proc.stdout), daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            self.reader.join(2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def traffic_table():
    """DRAM bytes per launch of the sweep's kernels from the committed ncu summary (profiles/), else {}."""
    path = os.path.join(ROOT, "profiles", "quantize_traffic.json")
    try:
        return json.load(open(path))
    except Exception:
        return {}


# ------------------------------------------------------------------------------------------------ GPU arm
def run_gpu(args):
    import torch
    import torch.distributed as dist
    import mxq
    from mxq import block, matmul, schedule

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    quant = {"mxquant": block.mxquant.quantize, "mxgemmini": block.mxgemmini.quantize, "ocp": block.ocp.quantize}
    V = synthetic(ROWS, COLS, 1000 + rank, dev)             # this rank's row shard of the global matrix
    runs = [(f, fmt, ax) for f in FAMILIES for fmt in FORMATS for ax in (0, 1)]

    def step():
        for f, fmt, ax in runs:
            quant[f](V, fmt, axis=ax)

    # -- device-resident sweep: per-launch CUDA events on the launching stream, then the whole timed loop
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    # per-launch durations: events around every launch of the first `nev` timed steps, on the launching stream
    nev = min(args.steps, 20)
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in runs]
           for _ in range(nev)]
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        barrier()
        start.record(stream)
        for s in range(args.steps):
            if s < nev:
                for (f, fmt, ax), (e0, e1) in zip(runs, evs[s]):
                    e0.record(stream)
                    quant[f](V, fmt, axis=ax)
                    e1.record(stream)
            else:
                step()
        end.record(stream)
        barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    per = {run: sum(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(nev)) / nev
           for i, run in enumerate(runs)}
    ms_step = ms / args.steps
    elems = ROWS * COLS
    total_bytes = BYTES_PER_ELEM * elems * len(runs) * world
    value = total_bytes / (ms_step * 1e-3) / 1e9

    # dominant kernel: the (family, axis) pair with the largest share of the sweep
    by_kernel = {}
    for (f, fmt, ax), t in per.items():
        by_kernel.setdefault((f, ax), []).append(t)
    dom, dom_ms = max(((k, sum(v)) for k, v in by_kernel.items()), key=lambda kv: kv[1])
    dom_avg = dom_ms / len(by_kernel[dom])
    hbm, peak_kind = peaks()
    achieved = BYTES_PER_ELEM * elems / (dom_avg * 1e-3) / 1e9
    kname = f"{dom[0]}/axis{dom[1]}"
    tr = traffic_table().get(kname)

    # -- the compact form: the OCP-grid families' sweep writing byte codes and E8M0 scales, through the C ABI (the
    # Python call reads its status word after every launch; the bench reads one at the end)
    import ctypes
    from mxq import _lib
    from mxq.block import mxgemmini as _mg, ocp as _oc
    pk_runs = [(f, fmt, ax) for f in ("mxgemmini", "ocp") for fmt in FORMATS for ax in (0, 1)]
    pk_st = torch.zeros(1, dtype=torch.int32, device=dev)
    pk_out = {}
    for f, fmt, ax in pk_runs:
        spec = (_mg.spec(fmt) if f == "mxgemmini" else _oc.spec(fmt))
        fe = spec.e + spec.m
        codes = torch.empty((ROWS, COLS // 2 if fe == 3 else COLS), dtype=torch.uint8, device=dev)
        scales = torch.empty((ROWS // 32, COLS) if ax == 0 else (ROWS, COLS // 32), dtype=torch.uint8, device=dev)
        lay = (1, ROWS, COLS) if ax == 0 else (ROWS, COLS, 1)
        pk_out[(f, fmt, ax)] = (spec, codes, scales, lay, fe)

    def pk_step():
        for run in pk_runs:
            spec, codes, scales, lay, _ = pk_out[run]
            _lib.call("mxq_block_quantize_packed", _lib.ptr(V), _lib.ptr(codes), _lib.ptr(scales), *lay, 32,
                      ctypes.byref(spec), _lib.ptr(pk_st), ctypes.c_void_p(stream.cuda_stream))

    for _ in range(args.warmup):
        pk_step()
    barrier()
    pk_steps = max(1, min(args.steps, 100))
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(pk_steps):
        pk_step()
    p1.record(stream)
    barrier()
    if int(pk_st.item()):
        raise RuntimeError("bench: the compact sweep reported a value the form cannot hold")
    pk_ms = max_over_ranks(p0.elapsed_time(p1)) / pk_steps
    pk_bytes = sum(elems * (4 + (0.5 if pk_out[r][4] == 3 else 1.0) + 1 / 32) for r in pk_runs) * world
    packed = {"workload": "compact form: block.{mxgemmini,ocp}.quantize_packed x 5 MX formats x axis {0,1} on the "
                          "same matrix (uint8 OCP codes, FP4 two a byte, E8M0 scale bytes), C ABI",
              "GB/s": round(pk_bytes / (pk_ms * 1e-3) / 1e9, 1),
              "Gelem/s": round(elems * len(pk_runs) * world / (pk_ms * 1e-3) / 1e9, 1),
              "float32 path Gelem/s": round(elems * len(runs) * world / (ms_step * 1e-3) / 1e9, 1),
              "ms_per_step": round(pk_ms, 4), "launches_per_step": len(pk_runs), "steps": pk_steps,
              "bytes_per_element": "4 read + 1 code (FP4 0.5) + 1/32 scale"}
    # -- the way back: dequantize (P, X) and the compact form's unpack / dequantize_packed, two formats x two axes
    def timed(fn, reps):
        fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps
    back = {"workload": "block.dequantize of the float32 codes, block.unpack and block.dequantize_packed of the "
                        "compact form, on the sweep's matrix (mxgemmini codes)",
            "bytes_per_element": "dequantize 8.125; unpack code + 4 + 1.125/32; dequantize_packed code + 4 + 1/32"}
    reps = max(1, min(args.steps, 50))
    for fmt in ("MXFP8_E4M3", "MXFP4"):
        for ax in (0, 1):
            spec, codes, scales, lay, fe = pk_out[("mxgemmini", fmt, ax)]
            cb = 0.5 if fe == 3 else 1.0
            P, X = quant["mxgemmini"](V, fmt, axis=ax)
            t_dq = timed(lambda: block.dequantize(P, X, axis=ax), reps)
            t_un = timed(lambda: block.unpack(codes, scales, fmt), reps)
            t_dp = timed(lambda: block.dequantize_packed(codes, scales, fmt, axis=ax), reps)
            back[f"{fmt}/axis{ax}"] = {
                "dequantize GB/s": round(BYTES_PER_ELEM * elems / (t_dq * 1e-3) / 1e9, 1),
                "unpack GB/s": round((cb + 4 + 1.125 / 32) * elems / (t_un * 1e-3) / 1e9, 1),
                "dequantize_packed GB/s": round((cb + 4 + 1 / 32) * elems / (t_dp * 1e-3) / 1e9, 1)}
            del P, X
    del pk_out

    # -- end to end through the public API with host tensors: each call streams its pinned host V through the
    # device and returns pinned host P, X (copies in and out on their own streams, overlapping the kernels); the
    # call returns once the results are on the host, so the host clock brackets the whole transfer
    Vh = V.cpu().pin_memory()
    e2e_steps = max(1, min(3, args.steps))

    def e2e_step():
        for f, fmt, ax in runs:
            quant[f](Vh, fmt, axis=ax)

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    barrier()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3) / e2e_steps
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    h2d = 4 * elems * len(runs) * world                     # whole job, like value
    d2h = (4 * elems + 4 * elems // 32) * len(runs) * world

    # -- config 3: the systolic GEMM, one 4096-column panel per rank
    gsteps = max(1, args.gemm_steps)
    gen = torch.Generator(device=dev).manual_seed(7)
    A = torch.randn(GEMM, GEMM, generator=gen, device=dev)
    B = torch.randn(GEMM, GEMM, generator=torch.Generator(device=dev).manual_seed(8 + rank), device=dev)
    arith = matmul.MXGEMMINI()

    def gemm():
        P_A, X_A = block.mxgemmini.quantize(A, "MXFP8_E4M3", axis=0)
        P_B, X_B = block.mxgemmini.quantize(B, "MXFP8_E4M3", axis=0)
        return matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL)

    for _ in range(max(1, args.warmup // 2)):
        gemm()
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(gsteps):
        gemm()
    g1.record(stream)
    barrier()
    gms = max_over_ranks(g0.elapsed_time(g1)) / gsteps
    gmacs = GEMM ** 3 * world / (gms * 1e-3) / 1e9

    # -- config 3's reducers on both operand formats (reducer kernel alone, CUDA events)
    def timed(fn, steps):
        fn()
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        barrier()
        return max_over_ranks(t0.elapsed_time(t1)) / steps

    red_out = {}
    for fmt in ("MXFP8_E4M3", "MXFP6_E2M3") if args.reducer_steps > 0 else ():
        P_A, X_A = block.mxgemmini.quantize(A, fmt, axis=0)
        P_B, X_B = block.mxgemmini.quantize(B, fmt, axis=0)
        reducers = {
            "systolic MXGEMMINI/HW_FINAL": lambda: matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL),
            "systolic MXQUANT(4,3)/HW_FINAL": lambda: matmul.systolic(P_A, X_A, P_B, X_B, matmul.MXQUANT(4, 3),
                                                                      schedule.HW_FINAL),
            "adder_tree MXGEMMINI [(4,4),(4,5),(4,6),(8,7)]": lambda: matmul.adder_tree(
                P_A, X_A, P_B, X_B, arith, [(4, 4), (4, 5), (4, 6), (8, 7)]),
            "anchor_tree MXGEMMINI (defaults)": lambda: matmul.anchor_tree(P_A, X_A, P_B, X_B, arith),
        }
        for name, fn in reducers.items():
            rms = timed(fn, args.reducer_steps)
            red_out[f"{fmt} {name}"] = {"GMAC/s": round(GEMM ** 3 * world / (rms * 1e-3) / 1e9, 1),
                                        "ms": round(rms, 3)}
        del P_A, X_A, P_B, X_B

    # -- config 1: the PR1 systolic GEMM (quantize x^T and W^T, systolic), 256 x 512 x 512
    extra = {}
    if args.extra_steps > 0:
        x = torch.randn(256, 512, generator=torch.Generator(device=dev).manual_seed(11), device=dev)
        W = torch.randn(512, 512, generator=torch.Generator(device=dev).manual_seed(12), device=dev)

        def pr1():
            PA1, XA1 = block.mxgemmini.quantize(x.t().contiguous(), "MXFP8_E4M3", axis=0)
            PB1, XB1 = block.mxgemmini.quantize(W.t().contiguous(), "MXFP8_E4M3", axis=0)
            return matmul.systolic(PA1, XA1, PB1, XB1, arith, schedule.HW_FINAL)

        ms1 = timed(pr1, 20 * args.extra_steps)
        extra["config 1: PR1 systolic 256x512x512 (quantize x^T, W^T + systolic)"] = {
            "GMAC/s": round(256 * 512 * 512 * world / (ms1 * 1e-3) / 1e9, 1), "us": round(ms1 * 1e3, 1)}

        # -- config 4: the LUT path on a 4096 x 4096 operand, column j ~ N(0, sigma_j^2), sigma_j = 2^U[-8, 8]
        from mxq import lut
        g4 = torch.Generator(device=dev).manual_seed(13 + rank)
        V4 = torch.randn(4096, 4096, generator=g4, device=dev) * torch.exp2(
            torch.rand(1, 4096, generator=g4, device=dev) * 16 - 8)
        n4 = V4.numel()
        for fmt in ("MXFP6_E3M2", "MXFP8_E4M3"):
            for G in (1, 3):
                ms4 = timed(lambda: block.lut.quantize(V4, fmt, 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23,
                                                       group=G, max_iters=50), args.extra_steps)
                extra[f"config 4: block.lut {fmt} G={G}"] = {
                    "GB/s": round(BYTES_PER_ELEM * n4 * world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 3)}
        P4 = block.mxgemmini.quantize(V4, "MXFP6_E3M2", 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
        T4 = lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=50)
        C4 = lut.encode(P4, "MXFP6_E3M2")
        for name, fn, bpe in (("lut.tables", lambda: lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=50), 4),
                              ("lut.pick", lambda: lut.pick(P4, T4, group=1), 12),
                              ("lut.finder", lambda: lut.finder(C4, T4, "MXFP6_E3M2", group=1), 16)):
            ms4 = timed(fn, args.extra_steps)
            extra[f"config 4: {name} MXFP6_E3M2 G=1"] = {
                "GB/s": round(bpe * n4 * world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 3)}
        del V4, P4, T4, C4

    # -- config 5: the MXLinear-patched Llama decoder (random init, std 0.02), 8 x 1024 tokens per GPU, one forward
    model_out = None
    if args.model_steps > 0:
        from functools import partial
        from transformers import LlamaConfig, LlamaForCausalLM
        from mxq import Scheme
        from mxq.nn import patch
        cfg = LlamaConfig(hidden_size=2048, intermediate_size=5632, num_hidden_layers=16, num_attention_heads=16,
                          num_key_value_heads=16, head_dim=128, vocab_size=32000, max_position_embeddings=1024,
                          initializer_range=0.02)
        torch.manual_seed(0)
        with torch.device(dev):
            model = LlamaForCausalLM(cfg).float().eval()
        q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
        sch = Scheme("hw_fp8", a=q8, b=q8, reduce=partial(matmul.systolic, arith=arith, schedule=schedule.HW_FINAL))
        handle = patch(model, [("lm_head", None), ("model.layers.*.self_attn", (sch, sch)), (torch.nn.Linear, sch)])
        ids = torch.randint(0, 32000, (8, 1024), generator=torch.Generator(device=dev).manual_seed(14 + rank),
                            device=dev)
        with torch.no_grad():
            msm = timed(lambda: model(ids).logits, args.model_steps)
        macs = 8 * 1024 * 16 * (4 * 2048 * 2048 + 3 * 2048 * 5632) + 8 * 16 * 16 * 2 * 1024 * 1024 * 128
        model_out = {"workload": "config 5: MXLinear-patched Llama (16 layers, hidden 2048, 16 heads x 128, FFN 5632, "
                                 "vocab 32000), batch 8 x 1024 tokens per GPU, one forward, every Linear but lm_head "
                                 "and the attention core through mxgemmini MXFP8_E4M3 + systolic MXGEMMINI/HW_FINAL",
                     "tokens/s": round(8 * 1024 * world / (msm * 1e-3), 1),
                     "emulated GMAC/s": round(macs * world / (msm * 1e-3) / 1e9, 1), "s_per_forward": round(msm / 1e3, 3),
                     "steps": args.model_steps}
        handle.revert()
        del model, handle, ids
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_rows, args.cpu_repeats)
    clocks = clk.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded config-2 distribution, generated on device)",
        "config": {"workload": "config 2: block.{mxquant,mxgemmini,ocp}.quantize x 5 MX formats x axis {0,1} on an "
                               "8192x8192 fp32 matrix per GPU", "rows_per_gpu": ROWS, "cols": COLS,
                   "launches_per_step": len(runs), "bytes_per_element": BYTES_PER_ELEM,
                   "l2": "inputs (256 MiB per matrix) larger than L2; no flush", "parallelism": f"rows x{world}"},
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1), "peak": hbm,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": tr},
        "kernels": {f"{f}/{fmt}/axis{ax}": round(BYTES_PER_ELEM * elems / (t * 1e-3) / 1e9, 1)
                    for (f, fmt, ax), t in sorted(per.items())},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": len(runs) * args.steps,
        "clocks": clocks,
        "systolic": {"metric": "bit-exact MX systolic-emulated GMAC/s", "value": round(gmacs, 2), "unit": "GMAC/s",
                     "workload": f"config 3: quantize A, B ({GEMM}x{GEMM} MXFP8_E4M3, block.mxgemmini) + "
                                 f"systolic MXGEMMINI/HW_FINAL {GEMM}^3 per GPU", "ms_per_gemm": round(gms, 3),
                     "steps": gsteps},
        "reducers": {"workload": f"config 3: {GEMM}^3 per GPU on MXFP8_E4M3 and MXFP6_E2M3 codes, reducer alone",
                     "steps": args.reducer_steps, **red_out},
        "configs_1_4": {"workload": "config 1 (PR1 GEMM, whole call) and config 4 (LUT path, 4096 x 4096 per GPU); "
                                    "GB/s counts 8.125 B/element for block.lut, 4 tables, 12 pick, 16 finder",
                        "steps": args.extra_steps, **extra},
        "model": model_out,
        "packed": packed,
        "dequantize": back,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- CPU oracle
def cpu_sweep_sample(rows, threads, repeats=1):
    """The sweep, `repeats` times, on a `rows` x 8192 slice with the CPU oracle; returns (GB/s, seconds)."""
    import oracle
    V = synthetic(rows, COLS, 1000).numpy()
    t0 = time.perf_counter()
    for _ in range(repeats):
        for f in FAMILIES:
            for fmt in FORMATS:
                for ax in (0, 1):
                    oracle.block_quantize(V, f, fmt, ax, threads=threads)
    dt = time.perf_counter() - t0
    return BYTES_PER_ELEM * V.size * 30 * repeats / dt / 1e9, dt


def cpu_baseline(rows, repeats):
    threads = os.cpu_count() or 1
    gbs, dt = cpu_sweep_sample(rows, threads, repeats)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"the same 30-run sweep, {repeats}x, on a {rows}x{COLS} matrix ({dt:.1f} s), CPU oracle (C "
                      "restatement of the reference algorithm), float32, all host threads"}


def run_reference(args):
    """The reference arm: the CPU restatement timed on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sweep_sample(args.ref_rows, threads)
    t0 = time.perf_counter()
    per = []
    for _ in range(args.steps):
        gbs, dt = cpu_sweep_sample(args.ref_rows, threads)
        per.append(dt)
    total = time.perf_counter() - t0
    value = BYTES_PER_ELEM * args.ref_rows * COLS * 30 * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded config-2 distribution)",
        "config": {"workload": "config 2: block.{mxquant,mxgemmini,ocp}.quantize x 5 MX formats x axis {0,1}",
                   "rows_per_step": args.ref_rows, "cols": COLS, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"each step: the 30-run sweep on a {args.ref_rows}x{COLS} row slice with the CPU "
                                   "oracle (the reference is pure Python/torch and is not installed on the GPU box; "
                                   "its measured CPU rate is 0.03-1.5 GB/s per quantizer)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mxq_b200", choices=["mxq_b200", "reference"])
    ap.add_argument("--gemm-steps", type=int, default=3)
    ap.add_argument("--reducer-steps", type=int, default=1, help="timed runs of each config-3 reducer (0: skip)")
    ap.add_argument("--extra-steps", type=int, default=3, help="timed runs of configs 1 and 4 (0: skip)")
    ap.add_argument("--model-steps", type=int, default=1, help="timed forwards of the config-5 model (0: skip)")
    ap.add_argument("--cpu-rows", type=int, default=ROWS, help="rows of the CPU-baseline matrix")
    ap.add_argument("--cpu-repeats", type=int, default=2, help="sweeps of the CPU-baseline matrix")
    ap.add_argument("--ref-rows", type=int, default=256, help="rows per reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
