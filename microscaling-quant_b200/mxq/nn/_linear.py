"""MXLinear: one nn.Linear computed through one Scheme, inference only (mxq/nn/_linear.py:37-80).

forward: x flattened to M×K float32, A = xᵀ, B = Wᵀ, Y = Aᵀ·B through the Scheme (its quantizers and reducer are CUDA
kernels), the float32 bias added, cast back to x's dtype. The weight codes are computed once (`refresh()` after the
weight changes); the tokens run `chunk` at a time, always whole multiples of the Scheme's `rows`. Output row m
depends on input row m only (LUT activations: on its 2^G-token group), so the chunk size changes no bit.
"""
from typing import Optional

import torch
from torch import nn

from ..scheme import Scheme

__all__ = ["MXLinear"]

#: tokens per call are kept under this many output elements (one reducer launch covers a whole chunk)
ELEMENTS_PER_STEP = 1 << 27


class MXLinear(nn.Module):
    def __init__(self, linear: nn.Linear, scheme: Scheme, chunk: Optional[int] = None,
                 cache_weights: bool = True):
        super().__init__()
        if chunk is not None and chunk < 1:
            raise ValueError(f"chunk must be >= 1, got {chunk}")
        if chunk is not None and chunk % scheme.rows:
            raise ValueError(f"chunk {chunk} must be a multiple of scheme {scheme.name!r} rows = {scheme.rows}")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.weight = linear.weight                   # the layer's own Parameter, not a copy
        self.bias = linear.bias
        self.scheme = scheme
        self.chunk = chunk
        self.cache_weights = cache_weights
        self.register_buffer("P_W", None, persistent=False)
        self.register_buffer("X_W", None, persistent=False)
        if cache_weights:
            self.refresh()

    @torch.no_grad()
    def refresh(self) -> None:
        """Recompute the cached weight codes and scales from `weight`."""
        self.P_W, self.X_W = self._codes()

    @torch.no_grad()
    def _codes(self):
        return self.scheme.b(self.weight.detach().float().t().contiguous())          # B = Wᵀ, K×N

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1]).float()                                      # M×K
        rows = self.scheme.rows
        step = self.chunk or max(rows, ELEMENTS_PER_STEP // self.out_features // rows * rows)
        P_W, X_W = (self.P_W, self.X_W) if self.cache_weights else self._codes()
        parts = [self.scheme.reduce(*self.scheme.a(p.t().contiguous()), P_W, X_W) for p in flat.split(step)]
        Y = parts[0] if len(parts) == 1 else torch.cat(parts)                         # M×N
        if self.bias is not None:
            Y = Y + self.bias.float()
        return Y.to(x.dtype).reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, scheme={self.scheme.name!r}"
