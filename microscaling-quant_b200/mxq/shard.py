"""The hot path across ranks, one process per GPU: every rank computes an independent slice of the output and one
`all_gather_into_tensor` reassembles it where the caller wants the whole result.

    quantize(block.mxgemmini.quantize, V, "MXFP8_E4M3", axis=0)       # rows (whole blocks) per rank
    reduce(matmul.systolic, P_A, X_A, P_B, X_B, arith, schedule)        # column panels of B per rank
    lut_tables(lut.tables, P, "MXFP6_E3M2", group=1)                    # column groups per rank
    rows(model_forward, ids)                                            # batch rows per rank

No slice depends on another: a block never straddles two ranks, a reducer panel keeps the whole K (the summation
order inside each output element is the specification, so K is never split), a LUT group keeps its columns. The
slices are balanced in whole units and every rank but the trailing ones holds a full slice, so the gathered
buffer, cut to length, is the result in order. With `gather=False` a rank gets its own slice and its range.

The compute callables are the package's own (or anything with their signature); the helpers only slice, call and
gather, on whatever device the callable returns (CUDA tensors with NCCL, CPU tensors with gloo). Without an
initialised process group they run the whole problem on this rank.
"""
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from .block._driver import _layout

__all__ = ["world", "split", "quantize", "reduce", "lut_tables", "rows", "GatherTarget", "quantize_gathered"]


def world(process_group=None) -> Tuple[int, int]:
    """(rank, world size) of this process in `process_group` (the default group), or (0, 1) without one."""
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(process_group), dist.get_world_size(process_group)


def split(n: int, parts: int, rank: int, multiple: int = 1) -> Tuple[int, int, int]:
    """(start, stop, capacity) of `rank`'s share of n items split into `parts` balanced runs of whole
    `multiple`-item units; capacity is the longest run, the slot each rank's result is padded to."""
    units = -(-n // multiple)
    per = -(-units // parts) if units else 0
    cap = per * multiple
    start = min(n, rank * cap)
    return start, min(n, start + cap), cap


def _gather(local: torch.Tensor, cap: int, dim: int, total: int, process_group) -> torch.Tensor:
    """Pad `local` along `dim` to `cap`, all-gather every rank's slot in rank order, cut to `total`."""
    rank, size = world(process_group)
    if size == 1:
        return local.narrow(dim, 0, total)
    local = local.movedim(dim, 0)
    slot = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    slot[:local.shape[0]] = local
    out = torch.empty((size * cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, slot.contiguous(), group=process_group)
    return out[:total].movedim(0, dim).contiguous()


def quantize(quantizer: Callable, V: torch.Tensor, fmt, axis: int = 0, block_size: int = 32, *,
             process_group=None, gather: bool = True, **kw):
    """A block quantizer's (P, X) with V's rows split across ranks. V viewed as [outer, len, inner] with blocks
    along len: outer > 1 splits whole outer slices, outer == 1 splits len at whole blocks. Every rank passes the
    same V (or at least its own rows, in place). Returns (P, X), or with gather=False (P_local, X_local, (start,
    stop)) in units of the split dimension."""
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    rank, size = world(process_group)
    if outer > 1:
        o0, o1, cap = split(outer, size, rank)
        Vl = V.reshape(outer, L, inner)[o0:o1]
        P, X = _run_quant(quantizer, Vl, fmt, 1, block_size, (o1 - o0, L, inner), (o1 - o0, nb, inner), V, kw)
        if not gather:
            return P, X, (o0, o1)
        P = _gather(P, cap, 0, outer, process_group)
        X = _gather(X, cap, 0, outer, process_group)
    else:
        r0, r1, cap = split(L, size, rank, block_size)
        Vl = V.reshape(L, inner)[r0:r1]
        nbl = -(-(r1 - r0) // block_size)
        P, X = _run_quant(quantizer, Vl, fmt, 0, block_size, (r1 - r0, inner), (nbl, inner), V, kw)
        if not gather:
            return P, X, (r0, r1)
        P = _gather(P, cap, 0, L, process_group)
        X = _gather(X, cap // block_size, 0, nb, process_group)
    xshape = list(V.shape)
    xshape[axis_] = nb
    return P.reshape(V.shape), X.reshape(xshape)


class GatherTarget:
    """Output buffers for quantize_gathered: P and X of the whole problem on every rank, in symmetric memory (each
    rank's buffers mapped into every other rank's address space over NVLink). Built collectively (every rank of the
    group, the same shapes); reused by every call with those shapes. A call overwrites them."""

    def __init__(self, shape, xshape, device, process_group=None):
        import torch.distributed._symmetric_memory as symm_mem
        group = process_group or dist.group.WORLD
        self.shape, self.xshape, self.device = tuple(shape), tuple(xshape), torch.device(device)
        self.P = symm_mem.empty(self.shape, dtype=torch.float32, device=self.device)
        self.X = symm_mem.empty(self.xshape, dtype=torch.float32, device=self.device)
        self._hp = symm_mem.rendezvous(self.P, group)
        self._hx = symm_mem.rendezvous(self.X, group)
        self.group = group
        self.rank, self.size = dist.get_rank(group), dist.get_world_size(group)
        # every rank's buffers as this process sees them (this rank's first), byte addresses
        order = [self.rank] + [r for r in range(self.size) if r != self.rank]
        self.p_ptrs = [int(self._hp.buffer_ptrs[r]) for r in order]
        self.x_ptrs = [int(self._hx.buffer_ptrs[r]) for r in order]

    def barrier(self):
        """Every rank's writes into every rank's buffers are complete and visible: a barrier of the group, which
        (NCCL) waits on each rank's earlier work on its current stream; bounded by the group's timeout."""
        dist.barrier(group=self.group)


def quantize_gathered(quantizer: Callable, V: torch.Tensor, fmt, axis: int = 0, block_size: int = 32, *,
                      target: GatherTarget, sync: bool = True, **kw):
    """quantize with V's rows split across the ranks, each rank's kernel writing its slice of P and X straight into
    every rank's `target` buffers over NVLink: the quantizer is the all-gather, no separate collective (no reference
    counterpart; quantize() does the same with an NCCL all-gather). `quantizer` is block.mxquant / mxgemmini / ocp's
    quantize and `kw` its options; blocks of 32 and the TMA kernel's layouts. Returns (target.P, target.X) after a
    barrier of the group; with sync=False the caller calls target.barrier() before any rank reads them (several
    calls can then share one barrier)."""
    import ctypes
    from . import _lib
    from .block import mxgemmini, mxquant, ocp
    module = {mxquant.quantize: mxquant, mxgemmini.quantize: mxgemmini, ocp.quantize: ocp}.get(quantizer)
    if module is None:
        raise ValueError("quantize_gathered: the quantizer must be block.mxquant, block.mxgemmini or block.ocp's "
                         "quantize")
    axis_, outer, L, inner, nb = _layout(V, axis, block_size)
    xshape = list(V.shape)
    xshape[axis_] = nb
    if target.shape != tuple(V.shape) or target.xshape != tuple(xshape):
        raise ValueError(f"quantize_gathered: target holds {target.shape} / {target.xshape}, the call needs "
                         f"{tuple(V.shape)} / {tuple(xshape)}")
    rank, size = target.rank, target.size
    spec = module.spec(fmt, **kw)
    v = V.contiguous()
    if outer > 1:                                   # whole outer slices
        o0, o1, _ = split(outer, size, rank)
        lay = (o1 - o0, L, inner)
        v_off, p_off, x_off = o0 * L * inner, o0 * L * inner, o0 * nb * inner
    else:                                           # whole blocks along len
        r0, r1, _ = split(L, size, rank, block_size)
        lay = (1, r1 - r0, inner)
        v_off, p_off, x_off = r0 * inner, r0 * inner, (r0 // block_size) * inner
    if lay[0] * lay[1] * lay[2] > 0:
        n = len(target.p_ptrs)
        ps = (ctypes.c_void_p * n)(*[p + 4 * p_off for p in target.p_ptrs])
        xs = (ctypes.c_void_p * n)(*[x + 4 * x_off for x in target.x_ptrs])
        _lib.run("mxq_block_quantize_multi", v.device, ctypes.c_void_p(v.data_ptr() + 4 * v_off), ps, xs, n,
                 *lay, block_size, ctypes.byref(spec))
    if sync:
        target.barrier()
    return target.P, target.X


def _run_quant(quantizer, Vl, fmt, axis, block_size, pshape, xshape, V, kw):
    if Vl.numel() == 0:                         # a trailing rank with nothing to do still joins the gather
        z = torch.zeros(pshape, dtype=torch.float32, device=V.device)
        return z, torch.zeros(xshape, dtype=torch.float32, device=V.device)
    return quantizer(Vl.contiguous(), fmt, axis=axis, block_size=block_size, **kw)


def reduce(reducer: Callable, P_A, X_A, P_B, X_B, *args, process_group=None, gather: bool = True, **kw):
    """A reducer's Y (M x N) with B's columns split into panels across ranks; every rank holds all of A and
    reduces over the whole K. Returns Y, or with gather=False (Y_local, (n0, n1))."""
    rank, size = world(process_group)
    N = P_B.shape[1]
    n0, n1, cap = split(N, size, rank)
    if n1 > n0:
        Y = reducer(P_A, X_A, P_B[:, n0:n1].contiguous(), X_B[:, n0:n1].contiguous(), *args, **kw)
    else:
        Y = torch.zeros((P_A.shape[1], 0), dtype=torch.float32, device=P_A.device)
    if not gather:
        return Y, (n0, n1)
    return _gather(Y, cap, 1, N, process_group)


def lut_tables(tables: Callable, P: torch.Tensor, fmt, group: int = 1, *, process_group=None, gather: bool = True,
               **kw):
    """lut.tables with P's columns split across ranks at whole groups of 2^group columns. Returns T, or with
    gather=False (T_local, (g0, g1)) in groups."""
    rank, size = world(process_group)
    n = P.shape[1]
    gs = 1 << group
    ngroups = -(-n // gs)
    c0, c1, cap = split(n, size, rank, gs)
    if c1 > c0:
        T = tables(P[:, c0:c1].contiguous(), fmt, group=group, **kw)
    else:
        T = torch.zeros((0, 16), dtype=torch.float32, device=P.device)
    if not gather:
        return T, (c0 // gs, -(-c1 // gs))
    return _gather(T, cap // gs, 0, ngroups, process_group)


def rows(fn: Callable[[torch.Tensor], torch.Tensor], x: torch.Tensor, *, process_group=None, gather: bool = True):
    """fn over x's leading rows split across ranks (a batch of sequences for a model, tokens for MXLinear); fn
    must treat rows independently. Returns fn(x), or with gather=False (fn(x_local), (r0, r1))."""
    rank, size = world(process_group)
    n = x.shape[0]
    r0, r1, cap = split(n, size, rank)
    y = fn(x[r0:r1]) if r1 > r0 else None
    if y is None:                               # learn the row shape from a one-row call, then send nothing real
        probe = fn(x[:1])
        y = probe[:0]
    if not gather:
        return y, (r0, r1)
    return _gather(y, cap, 0, n, process_group)
