"""Benchmark of the mxq B200 hot path (the driver's bench contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

Headline ("quantize GB/s"): the block-quantizer sweep. A step quantizes one float32
8192 x 8192 matrix -- N(0,1) x 2^U[-20,20] per row, 1% exact zeros, 0.1% float32-subnormal values -- with each of
block.mxquant / block.mxgemmini / block.ocp, each of the five MX formats, along axis 0 and axis 1: 30 fused kernel
launches. Throughput counts the algorithmic bytes of the reference's contract, 8.125 B per element (read V, write
P, write X once per 32 elements). Under torchrun every rank quantizes its own 8192-row shard of an (N * 8192)-row
matrix (weak scaling, no collective); the timed loop has nothing between launches, and each launch's own duration
comes from a separate, untimed pass with CUDA events around every launch.

Beside it, in the same JSON line:
  `parity`     the whole sweep (30 runs, P and X) compared bit for bit with the CPU oracle (oracle/, a C restatement
               of the reference) on the same matrix, inside the cpu_baseline leg (rank 0, N = 1)
  `sharded`    north_star's partitioning, strong scaling: ONE matrix / GEMM / operand / batch split across the N ranks
               by mxq.shard and reassembled by one NCCL all_gather_into_tensor inside the timed region -- config 2
               by rows, config 3's 4096^3 systolic GEMM by column panels of B, config 4's lut.tables by column groups,
               config 5's batch of 8 by rows -- with the gather's bytes and time, and rank 0's bit-for-bit check of
               the gathered result against its own whole-problem run
  `systolic`, `reducers`   config 3's reducers, each with a roofline against a fixed, spec-derived issue-slot count
               per emulated MAC (REDUCER_FLOORS)
  `configs_1_4`, `packed`, `dequantize`, `model`
  `e2e`        the sweep through the public API with a pinned host V per rank: every call streams V through the device
               in chunks and returns host P and X (copies in, kernels and copies out overlapped on three streams)
`--impl reference` is the reference arm: the CPU oracle on all host cores, rank 0 only, same metric, unit and config.
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
LEVELS = [(4, 4), (4, 5), (4, 6), (8, 7)]

# Issue slots per emulated MAC of each reducer datapath: the exact short forms of the kernels (their headers prove
# them) counted from the arithmetic's definition, every float32 multiply / add paired on sm_100's packed FP32
# instructions (half a slot per MAC), integer and compare / select steps one slot each, operand loads, register
# moves and the per-block work (scales, tile add: 1/16 of a MAC or less) not counted. A lower bound on the
# instructions, so MAC/s = 148 SMs x 4 schedulers x 32 lanes x clock / slots is an upper bound on the rate.
REDUCER_FLOORS = {
    # product 0.5 + 3-bit truncation mask 1 + snap onto the lane 1.0 + exact add 0.5 + lane RNE (exponent mask,
    # offset add, two adds: 1 + 1 + 1.0)
    "systolic MXGEMMINI/HW_FINAL": 6.0,
    # product 0.5 + qtorch rounding of the product (add, mask) 2 + fake-subnormal snap 1.0 and its compare / select 2
    # + lane add 0.5 + the lane's qtorch rounding 2 + its snap 1.0 and compare / select 2
    "systolic MXQUANT(4,3)/HW_FINAL": 11.0,
    # per 16 MACs: 16 products 8 + 16 masks 16; level 1: 8 folded snap-and-adds (3 adds each) 12 and 8 RNEs (2 integer
    # + 2 adds each) 16 + 8; level 2: 4 adds 2 + 4 RNEs 8 + 4; level 3: 2 adds 1 + 2 RNEs 4 + 2; level 4: one add
    # 0.5 and a bf16 pair conversion 0.5 -> 82 / 16
    "adder_tree MXGEMMINI [(4,4),(4,5),(4,6),(8,7)]": 82.0 / 16.0,
    # label sum 1 + label max 1 + product 0.5 + truncation mask 1 + scaling to the grid 0.5 + the keep step (sign
    # mask 1, round-toward-zero add and subtract 1.0) + the exact sum 0.5
    "anchor_tree MXGEMMINI (defaults)": 6.5,
}


def peaks():
    """Measured peaks (MEASURED_PEAKS.json, written by the driver), else the pool's fallback figures."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return {"hbm_gbs": float(p["hbm_gbs"]), "sm_max_mhz": float(p.get("sm_max_mhz", 1965.0)), "kind": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "sm_max_mhz": 1965.0, "kind": "fallback"}


def issue_peak_macs(slots_per_mac, mhz):
    """MAC/s when every SM scheduler issues one warp instruction per clock: 148 x 4 x 32 x clock / slots."""
    return 148 * 4 * 32 * mhz * 1e6 / slots_per_mac


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


def headline_config(world):
    """The `config` of the JSON line, the same for both arms."""
    return {"workload": "config 2: block.{mxquant,mxgemmini,ocp}.quantize x 5 MX formats x axis {0,1} on an "
                        "8192x8192 fp32 matrix per GPU", "rows_per_gpu": ROWS, "cols": COLS, "launches_per_step": 30,
            "bytes_per_element": BYTES_PER_ELEM, "l2": "inputs (256 MiB per matrix) larger than L2; no flush",
            "parallelism": f"rows x{world}"}


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
                                          "--format=csv,noheader,nounits", "-lms", "50"],
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
class Ranks:
    """This process's place in the job and the device-side timing helpers (every rank runs the same collectives in
    the same order)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all(self, ok):
        """True on every rank when `ok` is true on every rank."""
        if self.world == 1:
            return bool(ok)
        t = self.torch.tensor([0 if ok else 1], dtype=self.torch.int32, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return int(t.item()) == 0

    def timed(self, fn, steps):
        """fn() once untimed, then `steps` calls between CUDA events on the launching stream, barriers on both
        sides; the max over ranks of the mean ms per call."""
        torch = self.torch
        fn()
        self.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            fn()
        e1.record(self.stream)
        self.barrier()
        return self.max(e0.elapsed_time(e1)) / steps

    def check_waits(self, leg):
        from mxq import _lib
        self.torch.cuda.synchronize()
        _lib.check_waits()
        return leg


def same_bits(a, b):
    """Bit-identical device tensors (float32 or int64), shape included."""
    import torch
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    if a.dtype == torch.float32:
        return bool(torch.equal(a.view(torch.int32), b.view(torch.int32)))
    return bool(torch.equal(a, b))


def leg_sweep(R, args, quant, V, runs):
    """The headline: `steps` sweeps back to back between two events, nothing between the launches; then an
    untimed pass with events around every launch for each kernel's own duration."""
    torch = R.torch

    def step():
        for f, fmt, ax in runs:
            quant[f](V, fmt, axis=ax)

    for _ in range(args.warmup):
        step()
    R.barrier()
    est = R.timed(step, 2)                                     # ms per step, for the pre-roll below
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(R.local) as clk:
        for _ in range(int(300 / max(est, 1e-3)) + 1):          # ~0.3 s of untimed sweeps while the sampler starts,
            step()                                             # so every clock sample is taken under load
        R.barrier()
        start.record(R.stream)
        for _ in range(args.steps):
            step()
        end.record(R.stream)
        R.barrier()
    ms = R.max(start.elapsed_time(end))
    # the untimed pass: per-launch events (on the launching stream)
    nev = max(1, min(args.steps, 20))
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in runs]
           for _ in range(nev)]
    for s in range(nev):
        for (f, fmt, ax), (e0, e1) in zip(runs, evs[s]):
            e0.record(R.stream)
            quant[f](V, fmt, axis=ax)
            e1.record(R.stream)
    R.barrier()
    per = {run: sum(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(nev)) / nev for i, run in enumerate(runs)}
    R.check_waits("sweep")
    return ms / args.steps, per, clk.summary()


def leg_packed(R, args, V):
    """The compact form: the OCP-grid families' sweep writing byte codes and E8M0 scales, through the C ABI."""
    import ctypes
    torch = R.torch
    from mxq import _lib
    from mxq.block import mxgemmini as _mg, ocp as _oc
    pk_runs = [(f, fmt, ax) for f in ("mxgemmini", "ocp") for fmt in FORMATS for ax in (0, 1)]
    st = torch.zeros(1, dtype=torch.int32, device=R.dev)
    out = {}
    for f, fmt, ax in pk_runs:
        spec = (_mg.spec(fmt) if f == "mxgemmini" else _oc.spec(fmt))
        fe = spec.e + spec.m
        codes = torch.empty((ROWS, COLS // 2 if fe == 3 else COLS), dtype=torch.uint8, device=R.dev)
        scales = torch.empty((ROWS // 32, COLS) if ax == 0 else (ROWS, COLS // 32), dtype=torch.uint8, device=R.dev)
        lay = (1, ROWS, COLS) if ax == 0 else (ROWS, COLS, 1)
        out[(f, fmt, ax)] = (spec, codes, scales, lay, fe)

    def step():
        for run in pk_runs:
            spec, codes, scales, lay, _ = out[run]
            _lib.call("mxq_block_quantize_packed", _lib.ptr(V), _lib.ptr(codes), _lib.ptr(scales), *lay, 32,
                      ctypes.byref(spec), _lib.ptr(st), ctypes.c_void_p(R.stream.cuda_stream))

    for _ in range(args.warmup):
        step()
    steps = max(1, min(args.steps, 100))
    ms = R.timed(step, steps)
    if int(st.item()):
        raise RuntimeError(f"bench: the compact sweep reported status {int(st.item())}")
    R.check_waits("packed")
    elems = ROWS * COLS
    nbytes = sum(elems * (4 + (0.5 if out[r][4] == 3 else 1.0) + 1 / 32) for r in pk_runs) * R.world
    return out, {"workload": "compact form: block.{mxgemmini,ocp}.quantize_packed x 5 MX formats x axis {0,1} on the "
                             "same matrix (uint8 OCP codes, FP4 two a byte, E8M0 scale bytes), C ABI",
                 "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                 "Gelem/s": round(elems * len(pk_runs) * R.world / (ms * 1e-3) / 1e9, 1),
                 "ms_per_step": round(ms, 4), "launches_per_step": len(pk_runs), "steps": steps,
                 "bytes_per_element": "4 read + 1 code (FP4 0.5) + 1/32 scale"}


def leg_dequantize(R, args, quant, V, packed_out):
    """The way back: dequantize (P, X) and the compact form's unpack / dequantize_packed."""
    from mxq import block
    elems = ROWS * COLS
    res = {"workload": "block.dequantize of the float32 codes, block.unpack and block.dequantize_packed of the "
                       "compact form, on the sweep's matrix (mxgemmini codes)",
           "bytes_per_element": "dequantize 8.125; unpack code + 4 + 1.125/32; dequantize_packed code + 4 + 1/32"}
    reps = max(1, min(args.steps, 50))
    for fmt in ("MXFP8_E4M3", "MXFP4"):
        for ax in (0, 1):
            spec, codes, scales, lay, fe = packed_out[("mxgemmini", fmt, ax)]
            cb = 0.5 if fe == 3 else 1.0
            P, X = quant["mxgemmini"](V, fmt, axis=ax)
            t_dq = R.timed(lambda: block.dequantize(P, X, axis=ax), reps)
            t_un = R.timed(lambda: block.unpack(codes, scales, fmt), reps)
            t_dp = R.timed(lambda: block.dequantize_packed(codes, scales, fmt, axis=ax), reps)
            res[f"{fmt}/axis{ax}"] = {
                "dequantize GB/s": round(BYTES_PER_ELEM * elems * R.world / (t_dq * 1e-3) / 1e9, 1),
                "unpack GB/s": round((cb + 4 + 1.125 / 32) * elems * R.world / (t_un * 1e-3) / 1e9, 1),
                "dequantize_packed GB/s": round((cb + 4 + 1 / 32) * elems * R.world / (t_dp * 1e-3) / 1e9, 1)}
            del P, X
    return res


def leg_e2e(R, quant, V, runs):
    """The sweep through the public API with this rank's pinned host V; the calls return with P and X on the host,
    so the host clock brackets the whole transfer (max over ranks)."""
    Vh = V.cpu().pin_memory()
    steps = 2

    def step():
        for f, fmt, ax in runs:
            quant[f](Vh, fmt, axis=ax)

    step()
    R.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    R.barrier()
    ms = R.max((time.perf_counter() - t0) * 1e3) / steps
    elems = ROWS * COLS
    total = BYTES_PER_ELEM * elems * len(runs) * R.world
    h2d = 4 * elems * len(runs) * R.world
    d2h = (4 * elems + 4 * elems // 32) * len(runs) * R.world
    # the ceiling: the same bytes as plain pinned copies, host to device and back at once on two streams, every rank
    # at the same time (no kernel), host clock, max over ranks
    torch = R.torch
    Ph = torch.empty_like(Vh, pin_memory=True)
    Vd, Pd = torch.empty_like(V), torch.empty_like(V)
    s_in, s_out = torch.cuda.Stream(R.dev), torch.cuda.Stream(R.dev)
    reps = 10
    R.barrier()
    t0 = time.perf_counter()
    for _ in range(reps):
        with torch.cuda.stream(s_in):
            Vd.copy_(Vh, non_blocking=True)
        with torch.cuda.stream(s_out):
            Ph.copy_(Pd, non_blocking=True)
    s_in.synchronize()
    s_out.synchronize()
    R.barrier()
    cms = R.max((time.perf_counter() - t0) * 1e3) / reps
    ceiling = (4 * elems + 4 * elems) * R.world / (cms * 1e-3) / 1e9          # bytes moved per second, whole job
    moved = (h2d + d2h) / (ms * 1e-3) / 1e9
    return {"value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "pcie": {"moved_GB/s": round(moved, 1), "ceiling_GB/s": round(ceiling, 1),
                     "frac": round(moved / ceiling, 3),
                     "ceiling_kind": "pinned copies in and out at once on every rank, no kernel, host clock"}}


def gemm_operands(R, seed_b=8):
    torch = R.torch
    A = torch.randn(GEMM, GEMM, generator=torch.Generator(device=R.dev).manual_seed(7), device=R.dev)
    B = torch.randn(GEMM, GEMM, generator=torch.Generator(device=R.dev).manual_seed(seed_b), device=R.dev)
    return A, B


def reducer_roofline(name, gmacs, mhz):
    slots = REDUCER_FLOORS[name]
    peak = issue_peak_macs(slots, mhz) / 1e9
    return {"bound": "issue", "slots_per_mac": round(slots, 4), "achieved": round(gmacs, 1),
            "peak": round(peak, 1), "unit": "GMAC/s", "frac": round(gmacs / peak, 4),
            "clock_mhz": mhz, "peak_kind": "148 SMs x 4 schedulers x 32 lanes x clock / slots_per_mac"}


def leg_reducers(R, args, mhz):
    """config 3: the 4096^3 systolic GEMM with its quantization (per rank: its own B, weak), and the four reducers
    alone on both operand formats, each against its issue-slot roofline."""
    from mxq import block, matmul, schedule
    A, B = gemm_operands(R, 8 + R.rank)
    arith = matmul.MXGEMMINI()

    def gemm():
        P_A, X_A = block.mxgemmini.quantize(A, "MXFP8_E4M3", axis=0)
        P_B, X_B = block.mxgemmini.quantize(B, "MXFP8_E4M3", axis=0)
        return matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL)

    gms = R.timed(gemm, max(1, args.gemm_steps))
    gmacs = GEMM ** 3 * R.world / (gms * 1e-3) / 1e9
    systolic = {"metric": "bit-exact MX systolic-emulated GMAC/s", "value": round(gmacs, 2), "unit": "GMAC/s",
                "workload": f"config 3: quantize A, B ({GEMM}x{GEMM} MXFP8_E4M3, block.mxgemmini) + systolic "
                            f"MXGEMMINI/HW_FINAL {GEMM}^3 per GPU", "ms_per_gemm": round(gms, 3),
                "steps": max(1, args.gemm_steps),
                "roofline": reducer_roofline("systolic MXGEMMINI/HW_FINAL", gmacs / R.world, mhz)}
    reds = {"workload": f"config 3: {GEMM}^3 per GPU on MXFP8_E4M3 and MXFP6_E2M3 codes, reducer alone",
            "steps": args.reducer_steps}
    for fmt in ("MXFP8_E4M3", "MXFP6_E2M3") if args.reducer_steps > 0 else ():
        P_A, X_A = block.mxgemmini.quantize(A, fmt, axis=0)
        P_B, X_B = block.mxgemmini.quantize(B, fmt, axis=0)
        fns = {
            "systolic MXGEMMINI/HW_FINAL": lambda: matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL),
            "systolic MXQUANT(4,3)/HW_FINAL": lambda: matmul.systolic(P_A, X_A, P_B, X_B, matmul.MXQUANT(4, 3),
                                                                      schedule.HW_FINAL),
            "adder_tree MXGEMMINI [(4,4),(4,5),(4,6),(8,7)]": lambda: matmul.adder_tree(P_A, X_A, P_B, X_B, arith,
                                                                                        LEVELS),
            "anchor_tree MXGEMMINI (defaults)": lambda: matmul.anchor_tree(P_A, X_A, P_B, X_B, arith),
        }
        for name, fn in fns.items():
            rms = R.timed(fn, args.reducer_steps)
            g = GEMM ** 3 * R.world / (rms * 1e-3) / 1e9
            reds[f"{fmt} {name}"] = {"GMAC/s": round(g, 1), "ms": round(rms, 3),
                                     "roofline": reducer_roofline(name, g / R.world, mhz)}
        del P_A, X_A, P_B, X_B
    R.check_waits("reducers")
    return systolic, reds


def leg_configs_1_4(R, args):
    """config 1 (the PR1 GEMM, whole call) and config 4 (the LUT path on a 4096 x 4096 operand per rank)."""
    torch = R.torch
    from mxq import block, lut, matmul, schedule
    out = {}
    arith = matmul.MXGEMMINI()
    x = torch.randn(256, 512, generator=torch.Generator(device=R.dev).manual_seed(11), device=R.dev)
    W = torch.randn(512, 512, generator=torch.Generator(device=R.dev).manual_seed(12), device=R.dev)

    def pr1():
        PA1, XA1 = block.mxgemmini.quantize(x.t().contiguous(), "MXFP8_E4M3", axis=0)
        PB1, XB1 = block.mxgemmini.quantize(W.t().contiguous(), "MXFP8_E4M3", axis=0)
        return matmul.systolic(PA1, XA1, PB1, XB1, arith, schedule.HW_FINAL)

    ms1 = R.timed(pr1, 20 * args.extra_steps)
    out["config 1: PR1 systolic 256x512x512 (quantize x^T, W^T + systolic)"] = {
        "GMAC/s": round(256 * 512 * 512 * R.world / (ms1 * 1e-3) / 1e9, 1), "us": round(ms1 * 1e3, 1)}
    V4 = config4_operand(R, 13 + R.rank)
    n4 = V4.numel()
    for fmt in ("MXFP6_E3M2", "MXFP8_E4M3"):
        for G in (1, 3):
            ms4 = R.timed(lambda: block.lut.quantize(V4, fmt, 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23,
                                                     group=G, max_iters=50), args.extra_steps)
            out[f"config 4: block.lut {fmt} G={G}"] = {
                "GB/s": round(BYTES_PER_ELEM * n4 * R.world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 3)}
    # the same calls through the C ABI, back to back with preallocated outputs and one status read at the end: the
    # device's rate, without the Python call's preparation and its synchronous status check
    import ctypes
    from mxq import _lib
    from mxq.block import mxgemmini as _mg
    Pw, Xw = torch.empty_like(V4), torch.empty((4096 // 32, 4096), dtype=torch.float32, device=R.dev)
    st = torch.zeros(1, dtype=torch.int32, device=R.dev)
    stream = ctypes.c_void_p(R.stream.cuda_stream)
    for fmt in ("MXFP6_E3M2", "MXFP8_E4M3"):
        spec = _mg.spec(fmt, "rne", 2.0 ** -23)
        for G in (1, 3):
            ws = torch.empty(_lib.lib().mxq_block_lut_workspace(4096, 4096, 0, G), dtype=torch.uint8, device=R.dev)
            call = lambda: _lib.call("mxq_block_lut_quantize", _lib.ptr(V4), _lib.ptr(Pw), _lib.ptr(Xw), 4096, 4096,  # noqa: E731
                                     0, 32, ctypes.byref(spec), G, 50, _lib.ptr(ws), ws.numel(), _lib.ptr(st), stream)
            ms4 = R.timed(call, max(10, args.extra_steps))
            if int(st.item()):
                raise RuntimeError("bench: block.lut reported an off-grid code")
            out[f"config 4: block.lut {fmt} G={G} (C ABI, back to back)"] = {
                "GB/s": round(BYTES_PER_ELEM * n4 * R.world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 4)}
    P4 = block.mxgemmini.quantize(V4, "MXFP6_E3M2", 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
    T4 = lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=50)
    C4 = lut.encode(P4, "MXFP6_E3M2")
    Tw, Iw = torch.empty_like(T4), torch.empty((4096, 4096), dtype=torch.int64, device=R.dev)
    for name, fn, bpe in (
            ("lut.tables", lambda: _lib.call("mxq_lut_tables", _lib.ptr(P4), _lib.ptr(Tw), 4096, 4096, 4096, 1, 1, 50,
                                             3, 2, _lib.ptr(st), stream), 4),
            ("lut.pick", lambda: _lib.call("mxq_lut_pick", _lib.ptr(P4), _lib.ptr(T4), _lib.ptr(Iw), 4096, 4096, 4096,
                                           1, 1, 16, stream), 12),
            ("lut.finder", lambda: _lib.call("mxq_lut_finder", _lib.ptr(C4), _lib.ptr(T4), _lib.ptr(Iw), 4096, 4096, 1,
                                             3, 2, _lib.ptr(st), stream), 16)):
        ms4 = R.timed(fn, max(10, args.extra_steps))
        if int(st.item()):
            raise RuntimeError(f"bench: {name} reported a bad value")
        out[f"config 4: {name} MXFP6_E3M2 G=1 (C ABI, back to back)"] = {
            "GB/s": round(bpe * n4 * R.world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 4)}
    del Pw, Xw, Tw, Iw
    for name, fn, bpe in (("lut.tables", lambda: lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=50), 4),
                          ("lut.tables max_iters=0 (histogram and seeds, no Lloyd pass)",
                           lambda: lut.tables(P4, "MXFP6_E3M2", group=1, max_iters=0), 4),
                          ("lut.pick", lambda: lut.pick(P4, T4, group=1), 12),
                          ("lut.finder", lambda: lut.finder(C4, T4, "MXFP6_E3M2", group=1), 16)):
        ms4 = R.timed(fn, args.extra_steps)
        out[f"config 4: {name} MXFP6_E3M2 G=1"] = {
            "GB/s": round(bpe * n4 * R.world / (ms4 * 1e-3) / 1e9, 1), "ms": round(ms4, 3)}
    R.check_waits("configs 1 and 4")
    return out


def config4_operand(R, seed):
    """config 4's V: 4096 x 4096, column j ~ N(0, sigma_j^2), sigma_j = 2^U[-8, 8]."""
    torch = R.torch
    g = torch.Generator(device=R.dev).manual_seed(seed)
    return torch.randn(4096, 4096, generator=g, device=R.dev) * torch.exp2(
        torch.rand(1, 4096, generator=g, device=R.dev) * 16 - 8)


def llama(R):
    """config 5's model: the MXLinear-patched Llama decoder (random init, std 0.02)."""
    from functools import partial
    from transformers import LlamaConfig, LlamaForCausalLM
    from mxq import Scheme, block, matmul, schedule
    from mxq.nn import patch
    torch = R.torch
    cfg = LlamaConfig(hidden_size=2048, intermediate_size=5632, num_hidden_layers=16, num_attention_heads=16,
                      num_key_value_heads=16, head_dim=128, vocab_size=32000, max_position_embeddings=1024,
                      initializer_range=0.02)
    torch.manual_seed(0)
    with torch.device(R.dev):
        model = LlamaForCausalLM(cfg).float().eval()
    q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    sch = Scheme("hw_fp8", a=q8, b=q8, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(),
                                                       schedule=schedule.HW_FINAL))
    handle = patch(model, [("lm_head", None), ("model.layers.*.self_attn", (sch, sch)), (torch.nn.Linear, sch)])
    return model, handle


def leg_sharded(R, args, quant, runs):
    """north_star's partitioning, strong scaling, through mxq.shard: one problem split over the ranks and gathered
    by NCCL inside the timed region. Every rank builds the same inputs from the same seeds; rank 0 checks the
    gathered outputs bit for bit against its own whole-problem run (an untimed pass)."""
    torch = R.torch
    from mxq import block, lut, matmul, schedule, shard
    out = {"workload": "one problem split across the ranks by mxq.shard, reassembled by all_gather_into_tensor "
                       "(NCCL) in the timed region; gather_ms = total - compute-only (gather=False) time"}
    steps = max(1, min(args.steps, 10))

    # config 2: one 8192 x 8192 matrix, rows split (whole blocks along axis 0, whole rows along axis 1)
    V = synthetic(ROWS, COLS, 1000, R.dev)

    def sweep(gather):
        for f, fmt, ax in runs:
            shard.quantize(quant[f], V, fmt, axis=ax, gather=gather)

    t_all = R.timed(lambda: sweep(True), steps)
    t_cmp = R.timed(lambda: sweep(False), steps)
    ok = True
    for f, fmt, ax in runs:                                   # the parity pass: every rank gathers, rank 0 checks
        P, X = shard.quantize(quant[f], V, fmt, axis=ax)
        if R.rank == 0:
            Pw, Xw = quant[f](V, fmt, axis=ax)
            ok &= same_bits(P, Pw) and same_bits(X, Xw)
        del P, X
    ok = R.all(ok)
    gbytes = sum((ROWS * COLS + ROWS * COLS // 32) * 4 for _ in runs) * (R.world - 1) / max(1, R.world)
    out["config 2: sweep, rows split"] = {
        "GB/s": round(BYTES_PER_ELEM * ROWS * COLS * len(runs) / (t_all * 1e-3) / 1e9, 1),
        "ms_per_step": round(t_all, 3), "compute_ms": round(t_cmp, 3), "gather_ms": round(t_all - t_cmp, 3),
        "gather_bytes_received_per_rank": int(gbytes), "parity_vs_one_gpu": ok}
    # the same sweep with the gather fused into the quantizer: each rank's kernel writes its slice of P and X into
    # every rank's symmetric buffers over NVLink (no NCCL); one group barrier per step
    if R.world > 1:
        targets = {}
        for ax in (0, 1):
            xshape = [ROWS, COLS]
            xshape[ax] //= 32
            targets[ax] = shard.GatherTarget((ROWS, COLS), xshape, R.dev)

        def fused_sweep():
            for f, fmt, ax in runs:
                shard.quantize_gathered(quant[f], V, fmt, axis=ax, target=targets[ax], sync=False)
            targets[0].barrier()

        t_fused = R.timed(fused_sweep, steps)
        ok = True
        for f, fmt, ax in runs:                               # parity: every rank writes, rank 0 checks
            P, X = shard.quantize_gathered(quant[f], V, fmt, axis=ax, target=targets[ax])
            if R.rank == 0:
                Pw, Xw = quant[f](V, fmt, axis=ax)
                ok &= same_bits(P, Pw) and same_bits(X, Xw)
            targets[ax].barrier()                             # no rank writes the next run before rank 0 has read
        ok = R.all(ok)
        out["config 2: sweep, rows split, gather fused into the quantizer (NVLink stores)"] = {
            "GB/s": round(BYTES_PER_ELEM * ROWS * COLS * len(runs) / (t_fused * 1e-3) / 1e9, 1),
            "ms_per_step": round(t_fused, 3), "compute_ms (NCCL leg, gather=False)": round(t_cmp, 3),
            "nvlink_bytes_sent_per_rank": int(gbytes), "parity_vs_one_gpu": ok,
            "nvlink_roofline_ms": round(gbytes / 770e9 * 1e3, 3)}
        del targets
    del V

    # config 3: the 4096^3 systolic GEMM (MXGEMMINI / HW_FINAL), column panels of B
    A, B = gemm_operands(R)
    arith = matmul.MXGEMMINI()
    P_A, X_A = block.mxgemmini.quantize(A, "MXFP8_E4M3", axis=0)
    P_B, X_B = block.mxgemmini.quantize(B, "MXFP8_E4M3", axis=0)

    def gemm(gather):
        return shard.reduce(matmul.systolic, P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL, gather=gather)

    g_steps = max(1, args.gemm_steps)
    t_all = R.timed(lambda: gemm(True), g_steps)
    t_cmp = R.timed(lambda: gemm(False), g_steps)
    Y = gemm(True)
    ok = same_bits(Y, matmul.systolic(P_A, X_A, P_B, X_B, arith, schedule.HW_FINAL)) if R.rank == 0 else True
    ok = R.all(ok)
    out["config 3: systolic 4096^3, column panels"] = {
        "GMAC/s": round(GEMM ** 3 / (t_all * 1e-3) / 1e9, 1), "ms": round(t_all, 3), "compute_ms": round(t_cmp, 3),
        "gather_ms": round(t_all - t_cmp, 3),
        "gather_bytes_received_per_rank": int(GEMM * GEMM * 4 * (R.world - 1) / R.world), "parity_vs_one_gpu": ok}
    del A, B, P_A, X_A, P_B, X_B, Y

    # config 4: lut.tables by column groups (E3M2, G = 1 and 3)
    V4 = config4_operand(R, 13)
    P4 = block.mxgemmini.quantize(V4, "MXFP6_E3M2", 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
    for G in (1, 3):
        def tabs(gather):
            return shard.lut_tables(lut.tables, P4, "MXFP6_E3M2", group=G, max_iters=50, gather=gather)
        t_all = R.timed(lambda: tabs(True), max(1, args.extra_steps))
        t_cmp = R.timed(lambda: tabs(False), max(1, args.extra_steps))
        T = tabs(True)
        ok = same_bits(T, lut.tables(P4, "MXFP6_E3M2", group=G, max_iters=50)) if R.rank == 0 else True
        ok = R.all(ok)
        out[f"config 4: lut.tables MXFP6_E3M2 G={G}, column groups"] = {
            "GB/s": round(4 * P4.numel() / (t_all * 1e-3) / 1e9, 1), "ms": round(t_all, 3),
            "compute_ms": round(t_cmp, 3), "gather_ms": round(t_all - t_cmp, 3), "parity_vs_one_gpu": ok}
    del V4, P4
    R.check_waits("sharded")
    return out


def leg_model(R, args):
    """config 5: batch 8 x 1024 tokens split across the ranks by batch row (mxq.shard.rows), logits gathered; rank
    0 recomputes the last batch row on its own and compares (the north star's 1e-6 relative: the unquantized glue's
    kernels may sum in another order for another batch size)."""
    torch = R.torch
    from mxq import shard
    model, handle = llama(R)
    ids = torch.randint(0, 32000, (8, 1024), generator=torch.Generator(device=R.dev).manual_seed(14), device=R.dev)
    with torch.no_grad():
        fwd = lambda x: model(x).logits                                    # noqa: E731
        ms = R.timed(lambda: shard.rows(fwd, ids), args.model_steps)
        logits = shard.rows(fwd, ids)
        rel = 0.0
        if R.rank == 0:
            last = fwd(ids[-1:])
            rel = float((logits[-1:] - last).abs().max() / last.abs().max())
    ok = R.all(rel <= 1e-6)
    macs = 8 * 1024 * 16 * (4 * 2048 * 2048 + 3 * 2048 * 5632) + 8 * 16 * 16 * 2 * 1024 * 1024 * 128
    res = {"workload": "config 5: MXLinear-patched Llama (16 layers, hidden 2048, 16 heads x 128, FFN 5632, vocab "
                       "32000), one forward of batch 8 x 1024 tokens split across the ranks by batch row, logits "
                       "gathered; every Linear but lm_head and the attention core through mxgemmini MXFP8_E4M3 + "
                       "systolic MXGEMMINI/HW_FINAL (causal key blocks skipped per query chunk)",
           "tokens/s": round(8 * 1024 / (ms * 1e-3), 1), "emulated GMAC/s": round(macs / (ms * 1e-3) / 1e9, 1),
           "s_per_forward": round(ms / 1e3, 3), "steps": args.model_steps, "scaling": "strong",
           "gather_bytes_received_per_rank": int(8 * 1024 * 32000 * 4 * (R.world - 1) / R.world),
           "last_row_alone_rel_diff": rel, "parity_within_1e-6": ok}
    handle.revert()
    del model, handle, ids, logits
    torch.cuda.empty_cache()
    R.check_waits("model")
    return res


LEGS = ("sweep", "packed", "e2e", "reducers", "configs_1_4", "sharded", "model")


def run_gpu(args):
    import torch
    from mxq import block
    R = Ranks()
    legs = set(args.legs.split(",")) if args.legs else set(LEGS)
    quant = {"mxquant": block.mxquant.quantize, "mxgemmini": block.mxgemmini.quantize, "ocp": block.ocp.quantize}
    runs = [(f, fmt, ax) for f in FAMILIES for fmt in FORMATS for ax in (0, 1)]
    V = synthetic(ROWS, COLS, 1000 + R.rank, R.dev)            # this rank's row shard of the global matrix
    elems = ROWS * COLS
    pk = peaks()

    value = ms_step = achieved = kname = None
    per, clocks = {}, {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no timed sweep"]}
    if "sweep" in legs:
        ms_step, per, clocks = leg_sweep(R, args, quant, V, runs)
        value = BYTES_PER_ELEM * elems * len(runs) * R.world / (ms_step * 1e-3) / 1e9
        by_kernel = {}
        for (f, fmt, ax), t in per.items():
            by_kernel.setdefault((f, ax), []).append(t)
        dom, dom_ms = max(((k, sum(v)) for k, v in by_kernel.items()), key=lambda kv: kv[1])
        achieved = BYTES_PER_ELEM * elems / (dom_ms / len(by_kernel[dom]) * 1e-3) / 1e9
        kname = f"{dom[0]}/axis{dom[1]}"

    packed = back = e2e = systolic = reducers = sharded = model = None
    if "packed" in legs:
        packed_out, packed = leg_packed(R, args, V)
        back = leg_dequantize(R, args, quant, V, packed_out)
        del packed_out
    if "e2e" in legs:
        e2e = leg_e2e(R, quant, V, runs)
    mhz = clocks.get("sm_mhz") or pk["sm_max_mhz"]
    if "reducers" in legs:
        systolic, reducers = leg_reducers(R, args, mhz)
    extra = leg_configs_1_4(R, args) if args.extra_steps > 0 and "configs_1_4" in legs else {}
    if args.sharded and "sharded" in legs:
        sharded = leg_sharded(R, args, quant, runs)
    if args.model_steps > 0 and "model" in legs:
        model = leg_model(R, args)

    cpu = None
    if R.rank == 0 and R.world == 1 and not args.no_cpu_baseline and "sweep" in legs:
        cpu = cpu_baseline(V, quant, runs, args.cpu_repeats)
    if R.world > 1:
        R.dist.barrier()
        R.dist.destroy_process_group()
    if R.rank != 0:
        return
    line = {
        "metric": METRIC, "value": None if value is None else round(value, 2), "unit": "GB/s", "n_gpus": R.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None if ms_step is None else round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded config-2 distribution, generated on device)",
        "config": headline_config(R.world),
        "roofline": None if achieved is None else {
            "bound": "hbm", "kernel": kname, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
            "peak_kind": f"{pk['kind']} hbm_gbs", "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
            "traffic": traffic_table().get(kname),
            "timing": "each launch between CUDA events in an untimed pass after the timed loop"},
        "kernels": {f"{f}/{fmt}/axis{ax}": round(BYTES_PER_ELEM * elems / (t * 1e-3) / 1e9, 1)
                    for (f, fmt, ax), t in sorted(per.items())},
        "e2e": e2e,
        "gpu_launches": len(runs) * args.steps,
        "clocks": clocks,
        "systolic": systolic,
        "reducers": reducers,
        "configs_1_4": {"workload": "config 1 (PR1 GEMM, whole call) and config 4 (LUT path, 4096 x 4096 per GPU); "
                                    "GB/s counts 8.125 B/element for block.lut, 4 tables, 12 pick, 16 finder",
                        "steps": args.extra_steps, **extra},
        "sharded": sharded,
        "model": model,
        "packed": packed,
        "dequantize": back,
    }
    if cpu is not None:
        line["cpu_baseline"], line["parity"] = cpu
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- CPU oracle
def cpu_sweep_sample(Vh, threads):
    """The sweep once on the host matrix Vh with the CPU oracle; returns (GB/s, seconds)."""
    import oracle
    t0 = time.perf_counter()
    for f in FAMILIES:
        for fmt in FORMATS:
            for ax in (0, 1):
                oracle.block_quantize(Vh, f, fmt, ax, threads=threads)
    dt = time.perf_counter() - t0
    return BYTES_PER_ELEM * Vh.size * 30 / dt / 1e9, dt


def cpu_baseline(V, quant, runs, repeats):
    """The CPU oracle on the GPU's own matrix (copied to the host), all host threads, the sweep `repeats` times;
    the first time through, each run's oracle P and X are compared bit for bit with the GPU's (the parity flag)."""
    import oracle
    import torch
    threads = os.cpu_count() or 1
    Vh = V.cpu().numpy()
    oracle_s, bad = 0.0, []
    for f, fmt, ax in runs:
        t0 = time.perf_counter()
        Po, Xo = oracle.block_quantize(Vh, f, fmt, ax, threads=threads)
        oracle_s += time.perf_counter() - t0
        P, X = quant[f](V, fmt, axis=ax)
        torch.cuda.synchronize()
        P, X = P.cpu().numpy(), X.cpu().numpy()
        if not (np.array_equal(P.view(np.uint32), Po.view(np.uint32)) and
                np.array_equal(X.view(np.uint32), Xo.view(np.uint32))):
            bad.append(f"{f}/{fmt}/axis{ax}")
        del Po, Xo, P, X
    for _ in range(max(0, repeats - 1)):
        oracle_s += cpu_sweep_sample(Vh, threads)[1]
    gbs = BYTES_PER_ELEM * Vh.size * 30 * max(1, repeats) / oracle_s / 1e9
    cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": f"the same 30-run sweep, {max(1, repeats)}x, on the GPU's own 8192x8192 matrix ({oracle_s:.1f} s),"
                     " CPU oracle (C restatement of the reference algorithm), float32, all host threads"}
    parity = {"checked": "all 30 runs of the timed sweep, P and X, the whole 8192x8192 matrix, against the CPU oracle",
              "bit_exact": not bad, "mismatched_runs": bad}
    return cpu, parity


def run_reference(args):
    """The reference arm: the CPU restatement timed on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    Vh = synthetic(args.ref_rows, COLS, 1000).numpy()
    for _ in range(args.warmup):
        cpu_sweep_sample(Vh, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_sweep_sample(Vh, threads)
    total = time.perf_counter() - t0
    value = BYTES_PER_ELEM * args.ref_rows * COLS * 30 * args.steps / total / 1e9
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded config-2 distribution)", "config": headline_config(world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"each step: the 30-run sweep on a {args.ref_rows}x{COLS} row sample of the "
                                   "workload with the CPU oracle, all host threads (the reference is pure "
                                   "Python/torch and is not installed on the GPU box; its measured CPU rate is "
                                   "0.03-1.5 GB/s per quantizer)"},
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
    ap.add_argument("--no-sharded", dest="sharded", action="store_false", help="skip the strong-scaling leg")
    ap.add_argument("--cpu-repeats", type=int, default=2, help="sweeps of the CPU-baseline matrix")
    ap.add_argument("--ref-rows", type=int, default=256, help="rows per reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--legs", default="", help=f"comma-separated subset of {','.join(LEGS)} (default: all)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
