"""SwiGLU (aios/layers/activation.py:9-12) on the sm_100a kernel."""

from __future__ import annotations

import torch

from ..kernel import ops


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    return ops.silu_and_mul(x, out=out)


__all__ = ["silu_and_mul"]
