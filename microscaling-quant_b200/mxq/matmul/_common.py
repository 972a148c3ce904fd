"""Checks and helpers shared by every reducer (mxq/matmul/_common.py:8-34)."""
import math
from typing import Sequence, Tuple

import torch

from .. import _lib


def check_operands(P_A, X_A, P_B, X_B, block_size: int) -> Tuple[int, int, int]:
    """A: K x M with X_A: ceil(K/block_size) x M; B: K x N with X_B: ceil(K/block_size) x N; one device, float32.
    Returns (K, M, N)."""
    if any(t.ndim != 2 for t in (P_A, X_A, P_B, X_B)):
        raise ValueError(f"codes and scales must be 2-D, got ndim {[t.ndim for t in (P_A, X_A, P_B, X_B)]}")
    K, M = P_A.shape
    K_b, N = P_B.shape
    if K != K_b:
        raise ValueError(f"A is {K}×{M}, B is {K_b}×{N}: contraction lengths differ")
    nb = math.ceil(K / block_size)
    if tuple(X_A.shape) != (nb, M) or tuple(X_B.shape) != (nb, N):
        raise ValueError(f"scales must be {nb}×{M} and {nb}×{N} for block size {block_size}, "
                         f"got {tuple(X_A.shape)} and {tuple(X_B.shape)}")
    if len({t.device for t in (P_A, X_A, P_B, X_B)}) != 1:
        raise ValueError("codes and scales must be on one device")
    if any(t.dtype != torch.float32 for t in (P_A, X_A, P_B, X_B)):
        raise ValueError("codes and scales must be float32")
    return K, M, N


def check_schedule(schedule: Sequence[Tuple[int, int]], rows: int) -> None:
    """A schedule is fully defined when it has exactly one (e, m) row per accumulator position."""
    if len(schedule) != rows:
        raise ValueError(f"schedule has {len(schedule)} rows, reducer has {rows} accumulator positions")


def scale_map(X_A: torch.Tensor, X_B: torch.Tensor, g: int) -> torch.Tensor:
    """Outer product of block g's scales: the factor a finished block sum is multiplied by."""
    return X_A[g].unsqueeze(1) * X_B[g].unsqueeze(0)


def kernel_spec(arith, who: str):
    """The Arithmetic's kernel form, or an error for one built from arbitrary callables."""
    spec = getattr(arith, "spec", None)
    if spec is None:
        raise NotImplementedError(f"mxq_b200 {who}: Arithmetic {getattr(arith, 'name', arith)!r} has no kernel; "
                                  "build it with matmul.MXGEMMINI(...) or matmul.MXQUANT(...)")
    return spec


def operands(P_A, X_A, P_B, X_B):
    """The four operands contiguous on one CUDA device, and the device results go back to."""
    home = _lib.home(P_A)
    dev = _lib.device_for(P_A, X_A, P_B, X_B)
    return [_lib.on(t, dev) for t in (P_A, X_A, P_B, X_B)], dev, home


def _make_int_pairs(pairs):
    import ctypes
    es = (ctypes.c_int32 * max(1, len(pairs)))(*[int(e) for e, _ in pairs])
    ms = (ctypes.c_int32 * max(1, len(pairs)))(*[int(m) for _, m in pairs])
    return es, ms


_int_pairs = _lib.cached(_make_int_pairs)


def int_pairs(pairs):
    """A schedule as the two int32 arrays the entry points read (const): built once per schedule."""
    try:
        key = tuple((int(e), int(m)) for e, m in pairs)
    except (TypeError, ValueError):
        return _make_int_pairs(pairs)
    return _int_pairs(key)
