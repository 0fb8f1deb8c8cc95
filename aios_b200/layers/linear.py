"""Linear layers (aios/layers/linear.py:11-54) on the tcgen05 GEMM kernel."""

from __future__ import annotations

from collections.abc import Sequence

import torch

from .. import _lib
from ..kernel import ops
from .base import BaseOP


class Linear(BaseOP):
    def __init__(self, input_size: int, output_size: int, has_bias: bool = False):
        if has_bias:
            raise ValueError("the B200 linear kernels have no bias epilogue (the reference models use none)")
        self.weight = torch.empty(output_size, input_size)
        self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.weight)


class LinearQKVMerged(Linear):
    """One packed projection for Q, K and V: ``[Q | K | V]`` on the output dim."""

    def __init__(self, hidden_size: int, q_size: int, kv_size: int, has_bias: bool = False) -> None:
        super().__init__(hidden_size, q_size + 2 * kv_size, has_bias)
        self.q_size = q_size
        self.kv_size = kv_size


class LinearColParallelMerged(Linear):
    """Packed ``[gate | up]`` projection. ``forward`` keeps the reference output
    layout; ``forward_silu_mul`` runs the fused SwiGLU epilogue on a 64-row
    interleaved copy of the weight, built once when weights are loaded."""

    def __init__(self, input_size: int, output_sizes: Sequence[int], has_bias: bool = False) -> None:
        self.output_sizes = tuple(output_sizes)
        super().__init__(input_size, sum(self.output_sizes), has_bias)
        self._packed: torch.Tensor | None = None

    def on_weights_loaded(self) -> None:
        self._packed = None

    def packed_weight(self) -> torch.Tensor:
        if self._packed is None or self._packed.device != self.weight.device:
            if len(self.output_sizes) != 2 or self.output_sizes[0] != self.output_sizes[1]:
                raise ValueError("fused SwiGLU needs two equal output branches")
            self._packed = ops.pack_gate_up(self.weight)
        return self._packed

    def forward_silu_mul(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.packed_weight(), epilogue=_lib.EPI_SILU_MUL)
