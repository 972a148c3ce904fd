"""mxq.shard on CPU: the split rule, and gloo process groups of 2 and 3 ranks where each rank computes its slice
with the oracle (standing in for the rank's GPU) and the gathered result must equal the oracle's whole-problem
result bit for bit -- quantizers split by outer slices and by whole blocks, a reducer by column panels, LUT fits by
column groups, and batch rows. Three ranks give uneven splits and an empty trailing rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mxq import shard


def test_split():
    assert shard.split(10, 2, 0) == (0, 5, 5) and shard.split(10, 2, 1) == (5, 10, 5)
    assert shard.split(100, 3, 0, 32) == (0, 64, 64)        # 4 blocks over 3 ranks: 2, 2, 0 -> 64, 36, 0 rows
    assert shard.split(100, 3, 1, 32) == (64, 100, 64)
    assert shard.split(100, 3, 2, 32) == (100, 100, 64)
    assert shard.split(0, 4, 3) == (0, 0, 0)
    for n in range(0, 70):
        for parts in (1, 2, 3, 8):
            got = [shard.split(n, parts, r, 4)[:2] for r in range(parts)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            assert all(s % 4 == 0 or s == n for s, _ in got)     # whole units (an empty tail starts at n)


def _oracle_quantizer(family):
    import oracle

    def q(V, fmt, axis=0, block_size=32, **kw):
        P, X = oracle.block_quantize(V.numpy(), family, fmt, axis, block_size, **kw)
        return torch.from_numpy(P), torch.from_numpy(X)
    return q


def _oracle_systolic(P_A, X_A, P_B, X_B, arith, schedule):
    import oracle
    return torch.from_numpy(oracle.systolic(*(t.numpy() for t in (P_A, X_A, P_B, X_B)), arith, schedule))


def _oracle_tables(P, fmt, group=1, max_iters=50):
    import oracle
    return torch.from_numpy(oracle.lut_tables(P.numpy(), fmt, group, max_iters))


HW = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]


def _problems():
    rng = np.random.default_rng(4)
    V2 = (rng.standard_normal((100, 24)) * 2.0 ** rng.uniform(-6, 6, (100, 1))).astype(np.float32)
    V3 = rng.standard_normal((5, 40, 3)).astype(np.float32)
    A = rng.standard_normal((64, 12)).astype(np.float32)
    B = rng.standard_normal((64, 21)).astype(np.float32)
    L = (rng.standard_normal((64, 22)) * 2.0 ** rng.uniform(-4, 4, (1, 22))).astype(np.float32)
    return V2, V3, A, B, L


def _expected():
    import oracle
    V2, V3, A, B, L = _problems()
    out = {}
    for fam, fmt in (("mxquant", "MXFP8_E4M3"), ("ocp", "MXFP4")):
        for name, V, axis in (("v2a0", V2, 0), ("v2a1", V2, 1), ("v3a1", V3, 1), ("v3a0", V3, 0)):
            out[(fam, name)] = oracle.block_quantize(V, fam, fmt, axis)
    PA, XA = oracle.block_quantize(A, "mxgemmini", "MXFP8_E4M3", 0)
    PB, XB = oracle.block_quantize(B, "mxgemmini", "MXFP8_E4M3", 0)
    out["Y"] = oracle.systolic(PA, XA, PB, XB, oracle.arith_mxgemmini(), HW)
    PL = oracle.block_quantize(L, "mxgemmini", "MXFP6_E3M2", 0, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
    out["T"] = oracle.lut_tables(PL, "MXFP6_E3M2", 1, 50)
    return out, (PA, XA, PB, XB, PL)


def _check(got, want, what):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), what


def _rank_main(rank, size, port):
    import torch.distributed as dist
    import oracle
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        V2, V3, A, B, L = _problems()
        want, (PA, XA, PB, XB, PL) = _expected()
        fmts = {"mxquant": "MXFP8_E4M3", "ocp": "MXFP4"}
        for fam in ("mxquant", "ocp"):
            q = _oracle_quantizer(fam)
            for name, V, axis in (("v2a0", V2, 0), ("v2a1", V2, 1), ("v3a1", V3, 1), ("v3a0", V3, 0)):
                P, X = shard.quantize(q, torch.from_numpy(V), fmts[fam], axis=axis)
                _check(P, want[(fam, name)][0], f"{fam} {name} P")
                _check(X, want[(fam, name)][1], f"{fam} {name} X")
        Y = shard.reduce(_oracle_systolic, *(torch.from_numpy(t) for t in (PA, XA, PB, XB)),
                         oracle.arith_mxgemmini(), HW)
        _check(Y, want["Y"], "systolic panels")
        T = shard.lut_tables(_oracle_tables, torch.from_numpy(PL), "MXFP6_E3M2", group=1, max_iters=50)
        _check(T, want["T"], "lut tables")
        R = shard.rows(lambda x: x * 2.0 + 1.0, torch.arange(7 * 3, dtype=torch.float32).reshape(7, 3))
        _check(R, np.arange(21, dtype=np.float32).reshape(7, 3) * 2 + 1, "rows")
        Pl, Xl, (r0, r1) = shard.quantize(_oracle_quantizer("mxquant"), torch.from_numpy(V2), "MXFP8_E4M3",
                                          axis=0, gather=False)
        _check(Pl, want[("mxquant", "v2a0")][0][r0:r1], "local slice")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_single_process_is_whole_problem():
    want, (PA, XA, PB, XB, PL) = _expected()
    V2 = _problems()[0]
    P, X = shard.quantize(_oracle_quantizer("ocp"), torch.from_numpy(V2), "MXFP4", axis=0)
    _check(P, want[("ocp", "v2a0")][0], "P")
    _check(X, want[("ocp", "v2a0")][1], "X")


@pytest.mark.parametrize("size", [2, 3])
def test_gloo_ranks(size):
    mp.spawn(_rank_main, args=(size, _free_port()), nprocs=size, join=True)
