"""RMSNorm layers (aios/layers/norm.py:10-40) on the sm_100a kernels."""

from __future__ import annotations

from typing import Tuple

import torch

from ..kernel import ops
from .base import BaseOP


class RMSNorm(BaseOP):
    def __init__(self, size: int, eps: float = 1e-6) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)

    def forward_inplace(self, x: torch.Tensor) -> None:
        ops.rmsnorm(x, self.weight, self.eps, out=x)


class RMSNormFused(BaseOP):
    def __init__(self, size: int, eps: float = 1e-6) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(
        self, x: torch.Tensor, residual: torch.Tensor | None = None
    ) -> Tuple[torch.Tensor, torch.Tensor]:
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps), x
        ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
        return x, residual
