"""fp64_accum: the same codes and scales a reducer takes, with no rounding inside the multiply
(mxq/_fp64_accum.py:24-29): dequantize both operands in float32, then a float64 dot product per output, float32
out. One CUDA kernel (mxq_fp64_accum); the float64 sum runs in K order."""
import torch

from . import _lib
from .block import BLOCK

__all__ = ["fp64_accum"]


def fp64_accum(P_A: torch.Tensor, X_A: torch.Tensor, P_B: torch.Tensor, X_B: torch.Tensor,
               block_size: int = BLOCK) -> torch.Tensor:
    """Y = Aᵀ·B in float64, float32 out. A is K×M, B is K×N."""
    from .matmul._common import operands
    K, M = P_A.shape
    N = P_B.shape[1]
    (pa, xa, pb, xb), dev, home = operands(P_A, X_A, P_B, X_B)
    Y = torch.empty((M, N), dtype=torch.float32, device=dev)
    _lib.run("mxq_fp64_accum", dev, _lib.ptr(pa), _lib.ptr(xa), _lib.ptr(pb), _lib.ptr(xb), _lib.ptr(Y), K, M, N,
             block_size)
    return _lib.back(Y, home)
