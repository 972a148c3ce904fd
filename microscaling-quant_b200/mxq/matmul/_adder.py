"""The adder tree (mxq/matmul/_adder.py:42-71): `size` products at once, log2(size) levels of adjacent-pair
acc_add, level l in schedule[l]'s format; the root rescaled and tile_added. K tail: exact zeros. One CUDA kernel
per call (mxq_adder_tree)."""
import ctypes
from typing import Sequence, Tuple

import torch

from .. import _lib
from ..block import BLOCK
from ._common import check_operands, check_schedule, int_pairs, kernel_spec, operands
from ._arithmetic import Arithmetic

__all__ = ["adder_tree"]


def adder_tree(P_A: torch.Tensor, X_A: torch.Tensor, P_B: torch.Tensor, X_B: torch.Tensor,
               arith: Arithmetic, schedule: Sequence[Tuple[int, int]], size: int = 16,
               block_size: int = BLOCK) -> torch.Tensor:
    """Y = Aᵀ·B with each reduction of `size` products summed by a pairwise tree. `size` must be a power of two
    dividing `block_size`; `schedule` has one (e, m) per level."""
    K, M, N = check_operands(P_A, X_A, P_B, X_B, block_size)
    levels = size.bit_length() - 1
    if size < 2 or (1 << levels) != size:
        raise ValueError(f"size {size} must be a power of two >= 2")
    if block_size % size != 0:
        raise ValueError(f"size {size} must divide block size {block_size}")
    check_schedule(schedule, levels)
    spec = kernel_spec(arith, "adder_tree")
    (pa, xa, pb, xb), dev, home = operands(P_A, X_A, P_B, X_B)
    Y = torch.empty((M, N), dtype=torch.float32, device=dev)
    es, ms = int_pairs(schedule)
    c = spec.c_struct()
    _lib.run("mxq_adder_tree", dev, _lib.ptr(pa), _lib.ptr(xa), _lib.ptr(pb), _lib.ptr(xb), _lib.ptr(Y), K, M, N,
             block_size, size, ctypes.byref(c), es, ms)
    return _lib.back(Y, home)
