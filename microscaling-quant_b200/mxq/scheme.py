"""mxq.scheme — one explicit chain for one matmul (mxq/scheme.py:40-68): how each operand becomes codes and how
the codes are multiplied.

    Scheme(name, a, b, reduce, rows=1, block_size=32)
        a(V) -> (P, X), b(V) -> (P, X), reduce(P_A, X_A, P_B, X_B) -> Y
    Scheme.matmul(A, B) -> Y = Aᵀ·B
"""
import math
from dataclasses import dataclass
from typing import Callable, Tuple

import torch

from .block import BLOCK

__all__ = ["Scheme"]

Tensor = torch.Tensor
Quantizer = Callable[[Tensor], Tuple[Tensor, Tensor]]
Reducer = Callable[[Tensor, Tensor, Tensor, Tensor], Tensor]


@dataclass(frozen=True)
class Scheme:
    name: str
    a: Quantizer
    b: Quantizer
    reduce: Reducer
    rows: int = 1
    block_size: int = BLOCK

    def __post_init__(self):
        for field in ("rows", "block_size"):
            v = getattr(self, field)
            if not isinstance(v, int) or isinstance(v, bool) or v < 1:
                raise ValueError(f"Scheme: {field} {v!r} must be a positive integer")

    def check_scales(self, X: Tensor, K: int, operand: str) -> None:
        """X must hold one row of scales per `block_size` of K."""
        if X.shape[0] != math.ceil(K / self.block_size):
            raise ValueError(f"Scheme {self.name!r}: {operand} has {X.shape[0]} scale rows for K = {K}, "
                             f"block_size {self.block_size} needs {math.ceil(K / self.block_size)}; "
                             "the Scheme's block_size and its quantizer's disagree")

    def matmul(self, A: Tensor, B: Tensor) -> Tensor:
        """Y = Aᵀ·B for A: K×M and B: K×N."""
        P_A, X_A = self.a(A)
        P_B, X_B = self.b(B)
        self.check_scales(X_A, A.shape[0], "a")
        self.check_scales(X_B, B.shape[0], "b")
        return self.reduce(P_A, X_A, P_B, X_B)
