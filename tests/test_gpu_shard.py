"""mxq.shard on real GPUs with NCCL (skipped with fewer than two devices): one process per GPU, each computing its
slice of config-2, config-3 and config-4 style problems on its own device, the slices reassembled by NCCL
all_gather_into_tensor -- and, for the quantizers, by the fused form, whose kernel writes each rank's slice into every
rank's symmetric buffers over NVLink; every rank checks the gathered result bit for bit against the same problem
computed whole on its own GPU. Run on 2 GPUs (and on more when they are there, up to 4)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HW = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _same(a, b):
    return a.shape == b.shape and a.dtype == b.dtype and bool(torch.equal(a.view(torch.int32), b.view(torch.int32)))


def _rank_main(rank, size, port, errors):
    import datetime
    import torch.distributed as dist
    from mxq import block, lut, matmul, schedule, shard
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=size, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    bad = []
    try:
        g = torch.Generator(device=dev).manual_seed(3)
        V = (torch.randn(1000, 768, generator=g, device=dev) *
             torch.exp2(torch.rand(1000, 1, generator=g, device=dev) * 30 - 15))   # 1000 rows: a ragged last block
        for f, q in (("mxquant", block.mxquant.quantize), ("ocp", block.ocp.quantize)):
            for ax in (0, 1):
                P, X = shard.quantize(q, V, "MXFP6_E2M3", axis=ax)
                Pw, Xw = q(V, "MXFP6_E2M3", axis=ax)
                if not (_same(P, Pw) and _same(X, Xw)):
                    bad.append(f"quantize {f} axis {ax}")
        A = torch.randn(512, 200, generator=g, device=dev)
        B = torch.randn(512, 333, generator=g, device=dev)
        PA, XA = block.mxgemmini.quantize(A, "MXFP8_E4M3", axis=0)
        PB, XB = block.mxgemmini.quantize(B, "MXFP8_E4M3", axis=0)
        for name, red, extra in (("systolic", matmul.systolic, (matmul.MXGEMMINI(), schedule.HW_FINAL)),
                                 ("adder", matmul.adder_tree, (matmul.MXGEMMINI(), [(4, 4), (4, 5), (4, 6), (8, 7)]))):
            Y = shard.reduce(red, PA, XA, PB, XB, *extra)
            if not _same(Y, red(PA, XA, PB, XB, *extra)):
                bad.append(f"reduce {name}")
        L = torch.randn(256, 90, generator=g, device=dev) * torch.exp2(torch.rand(1, 90, generator=g, device=dev) * 8)
        PL = block.mxgemmini.quantize(L, "MXFP6_E3M2", 0, 32, rounding_mode="rne", scale_floor=2.0 ** -23)[0]
        for G in (1, 3):
            T = shard.lut_tables(lut.tables, PL, "MXFP6_E3M2", group=G, max_iters=20)
            if not _same(T, lut.tables(PL, "MXFP6_E3M2", group=G, max_iters=20)):
                bad.append(f"lut.tables G={G}")
        # the fused form: each rank's quantizer writes its slice into every rank's symmetric buffers over NVLink
        for f, q in (("mxgemmini", block.mxgemmini.quantize), ("mxquant", block.mxquant.quantize),
                     ("ocp", block.ocp.quantize)):
            for ax in (0, 1):
                xshape = list(V.shape)
                xshape[ax] = -(-V.shape[ax] // 32)
                target = shard.GatherTarget(V.shape, xshape, dev)
                for call in range(2):                        # the target is reused
                    P, X = shard.quantize_gathered(q, V, "MXFP8_E4M3", axis=ax, target=target)
                    Pw, Xw = q(V, "MXFP8_E4M3", axis=ax)
                    if not (_same(P, Pw) and _same(X, Xw)):
                        bad.append(f"quantize_gathered {f} axis {ax} call {call}")
                del target
        R = shard.rows(lambda x: x * 3.0 - 1.0, torch.arange(45, dtype=torch.float32, device=dev).reshape(9, 5))
        if not _same(R, torch.arange(45, dtype=torch.float32, device=dev).reshape(9, 5) * 3.0 - 1.0):
            bad.append("rows")
        dist.barrier()
    except Exception as e:                                    # report it; the other ranks end at their timeout
        bad.append(repr(e))
    finally:
        dist.destroy_process_group()
    errors.put((rank, bad))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_nccl_shards_equal_whole_problem():
    size = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, size, port, errors)) for r in range(size)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    results = [errors.get(timeout=10) for _ in procs]
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert all(not bad for _, bad in results), results
