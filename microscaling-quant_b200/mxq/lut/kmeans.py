"""Fitting the tables and picking indices for a K×n tensor of block codes, one table per 2^G columns
(mxq/lut/kmeans.py:46-146):

    T = tables(P, fmt, group=G, max_iters=50)   ceil(n / 2^G) × SIZE values, each row ascending
    I = pick(P, T, group=G)                     K×n int64: each code's nearest entry, ties to the lower index
    P_lut = lookup(I, T, group=G)

tables: the group's distinct codes weighted by their counts; 16 or fewer are the centres, else quantile seeds and
weighted Lloyd passes (float64, stop when two passes agree to numpy.allclose or after max_iters); each centre
snapped to the nearest finder-safe value; padded with unused values of smallest magnitude; sorted. One CUDA kernel
(mxq_lut_tables): a CTA per panel of groups, the histograms in shared memory, a warp per group fit.
"""
import torch

from .. import _lib
from .formats import SIZE, _format

__all__ = ["tables", "pick", "lookup"]


def _check(P: torch.Tensor, group: int) -> int:
    if P.ndim != 2:
        raise ValueError(f"mxq.lut: expects a K×n tensor, got shape {tuple(P.shape)}")
    if not isinstance(group, int) or isinstance(group, bool) or group < 0:
        raise ValueError(f"mxq.lut: group {group!r} must be a non-negative integer")
    return (P.shape[1] + (1 << group) - 1) >> group


def _check_tables(T: torch.Tensor, ng: int, n: int, group: int, who: str) -> None:
    if T.ndim != 2 or T.shape[0] != ng or T.shape[1] < 2:
        raise ValueError(f"mxq.lut.{who}: {n} columns at group {group} need ({ng}, width) tables with width >= 2, "
                         f"got {tuple(T.shape)}")


def _strides(P: torch.Tensor):
    """A K×n operand in place: row-major (sk = n, sj = 1) or the transpose of a row-major n×K (sk = 1, sj = K)."""
    K, n = P.shape
    if P.is_contiguous():
        return P, n, 1
    if P.t().is_contiguous():
        return P, 1, K
    return P.contiguous(), n, 1


def tables(P: torch.Tensor, fmt, *, group: int, max_iters: int) -> torch.Tensor:
    """One SIZE-entry table per 2^group columns of P (K×n block codes of fmt); the last covers the columns left."""
    f = _format(fmt)
    ng = _check(P, group)
    if not isinstance(max_iters, int) or isinstance(max_iters, bool) or max_iters < 0:
        raise ValueError(f"mxq.lut: max_iters {max_iters!r} must be a non-negative integer")
    home = _lib.home(P)
    dev = _lib.device_for(P)
    p = P.detach().to(device=dev, dtype=torch.float32)
    p, sk, sj = _strides(p)
    K, n = P.shape
    T = torch.empty((ng, SIZE), dtype=torch.float32, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.run("mxq_lut_tables", dev, _lib.ptr(p), _lib.ptr(T), K, n, sk, sj, group, max_iters, f.e, f.m, _lib.ptr(st))
    if int(st.item()):
        raise ValueError(f"mxq.lut: P holds a value that is not a {f.name} code; quantize it first")
    return _lib.back(T, home)


def pick(P: torch.Tensor, T: torch.Tensor, *, group: int) -> torch.Tensor:
    """Each code's nearest entry in its column group's table, ties to the lower index. K×n int64."""
    ng = _check(P, group)
    _check_tables(T, ng, P.shape[1], group, "pick")
    home = _lib.home(P)
    dev = _lib.device_for(P, T)
    p = P.detach().to(device=dev, dtype=torch.float32)
    p, sk, sj = _strides(p)
    t = _lib.on(T, dev)
    K, n = P.shape
    I = torch.empty((K, n), dtype=torch.int64, device=dev)
    _lib.run("mxq_lut_pick", dev, _lib.ptr(p), _lib.ptr(t), _lib.ptr(I), K, n, sk, sj, group, t.shape[1])
    return _lib.back(I, home)


def pick_lookup(P: torch.Tensor, T: torch.Tensor, *, group: int) -> torch.Tensor:
    """lookup(pick(P, T), T) in one pass, written in P's own layout (block.lut's last step)."""
    ng = _check(P, group)
    _check_tables(T, ng, P.shape[1], group, "pick")
    home = _lib.home(P)
    dev = _lib.device_for(P, T)
    p = P.detach().to(device=dev, dtype=torch.float32)
    p, sk, sj = _strides(p)
    t = _lib.on(T, dev)
    K, n = P.shape
    out = torch.empty_like(p)
    _lib.run("mxq_lut_pick_lookup", dev, _lib.ptr(p), _lib.ptr(t), _lib.ptr(out), K, n, sk, sj, group, t.shape[1])
    return _lib.back(out, home)


def lookup(I: torch.Tensor, T: torch.Tensor, *, group: int) -> torch.Tensor:
    """The values the indices name: K×n float32."""
    ng = _check(I, group)
    _check_tables(T, ng, I.shape[1], group, "lookup")
    home = _lib.home(I)
    dev = _lib.device_for(I, T)
    i = _lib.on(I, dev, torch.int64)
    t = _lib.on(T, dev)
    K, n = I.shape
    out = torch.empty((K, n), dtype=torch.float32, device=dev)
    _lib.run("mxq_lut_lookup", dev, _lib.ptr(i), _lib.ptr(t), _lib.ptr(out), K, n, group, t.shape[1])
    return _lib.back(out, home)
