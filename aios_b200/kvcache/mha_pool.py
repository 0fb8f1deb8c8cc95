"""Paged MHA KV cache (replaces aios/kvcache/mha_pool.py:8-68).

Same buffer layout as the reference, ``[2, layers, pages, page_size, Hkv, d]``,
now for page_size 1 (the reference's only mode: every page is one token slot)
or 16. Token slot s of a layer is row s of the flattened ``[pages * page_size,
Hkv, d]`` view, which is what every kernel indexes.
"""

from __future__ import annotations

import torch

from ..kernel.ops import store_cache
from .base import BaseKVCache

SUPPORTED_PAGE_SIZES = (1, 16)


class MHAKVCache(BaseKVCache):
    def __init__(
        self,
        num_kv_heads: int,
        num_layers: int,
        head_dim: int,
        num_pages: int,
        page_size: int,
        dtype: torch.dtype,
        device: torch.device,
    ) -> None:
        if device.type != "cuda":
            raise ValueError("MHAKVCache lives in CUDA device memory")
        if page_size not in SUPPORTED_PAGE_SIZES:
            raise ValueError(f"page_size must be one of {SUPPORTED_PAGE_SIZES}")
        if dtype != torch.bfloat16:
            raise ValueError("the B200 kernels store the KV cache in bf16")
        self._kv_buffer = torch.zeros(
            (2, num_layers, num_pages, page_size, num_kv_heads, head_dim), device=device, dtype=dtype
        )
        self._num_layers = num_layers
        self._k_buffer = self._kv_buffer[0]
        self._v_buffer = self._kv_buffer[1]
        self._device = device
        self.page_size = page_size
        self.num_pages = num_pages
        self.num_slots = num_pages * page_size
        self._storage_shape = (num_pages * page_size, num_kv_heads, head_dim)

    def k_cache(self, index: int) -> torch.Tensor:
        return self._k_buffer[index]

    def v_cache(self, index: int) -> torch.Tensor:
        return self._v_buffer[index]

    def k_slots(self, index: int) -> torch.Tensor:
        """Layer `index` keys as [slots, Hkv, d]."""
        return self._k_buffer[index].view(self._storage_shape)

    def v_slots(self, index: int) -> torch.Tensor:
        return self._v_buffer[index].view(self._storage_shape)

    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer_id: int) -> None:
        store_cache(self.k_slots(layer_id), self.v_slots(layer_id), out_loc, k, v)

    @property
    def device(self) -> torch.device:
        return self._device

    @property
    def dtype(self) -> torch.dtype:
        return self._kv_buffer.dtype

    @property
    def num_layers(self) -> int:
        return self._num_layers
