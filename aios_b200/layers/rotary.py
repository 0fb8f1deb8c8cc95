"""RoPE tables (aios/layers/rotary.py:8-29).

The fp32 cos/sin caches are computed on the CPU with the reference's formula
(theta^(-2i/d), ``cat(freqs, freqs)``); the kernels read bf16 copies, the same
values ``apply_rotary_pos_emb`` casts them to.
"""

from __future__ import annotations

import torch

from .base import StateLessOP


class RotaryEmbedding(StateLessOP):
    def __init__(self, head_dim: int, max_position_embeddings: int, base: float = 1000000.0):
        with torch.device("cpu"):
            inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
            t = torch.arange(max_position_embeddings, dtype=torch.float32)
            freqs = torch.outer(t, inv_freq)
            emb = torch.cat((freqs, freqs), dim=-1)
            self._cos_cache = emb.cos()
            self._sin_cache = emb.sin()
        self._cos_bf16: torch.Tensor | None = None
        self._sin_bf16: torch.Tensor | None = None

    def forward(self, position_ids: torch.Tensor):
        cos = self._cos_cache[position_ids]
        sin = self._sin_cache[position_ids]
        return cos.unsqueeze(1), sin.unsqueeze(1)

    def set_device(self, device: torch.device) -> None:
        self._cos_cache = self._cos_cache.to(device)
        self._sin_cache = self._sin_cache.to(device)
        self._cos_bf16 = self._cos_cache.to(torch.bfloat16).contiguous()
        self._sin_bf16 = self._sin_cache.to(torch.bfloat16).contiguous()

    def tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        """bf16 [max_pos, head_dim] device tables used by the fused kernels."""
        if self._cos_bf16 is None:
            raise RuntimeError("RotaryEmbedding.set_device() has not been called")
        return self._cos_bf16, self._sin_bf16
