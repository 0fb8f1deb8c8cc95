"""Free-slot FIFO of the paged KV pool (replaces aios/scheduler/cache.py:9-51).

The free list lives on the device as a ring of ``num_pages`` int32 ids with
logical head/tail counters mirrored here on the host: ``allocate(n)`` hands out
the first n free ids, ``_free`` appends at the tail, so ids come back in exactly
the reference's FIFO order (initially ``arange(num_pages)``). The CandidateGroup
step kernel allocates from the same ring on the device and reports the new head
back through :meth:`advance_head`.

With ``page_size`` 1 an id is a token slot (the reference layout); with 16 an id
is a page of 16 consecutive token slots.
"""

from __future__ import annotations

import torch

from ..core import Req
from ..kernel import ops


class CacheManager:
    def __init__(self, device: torch.device, num_pages: int, page_size: int = 1):
        if device.type != "cuda":
            raise ValueError("CacheManager keeps its free list on a CUDA device")
        if num_pages < 1:
            raise ValueError("num_pages must be positive")
        self.device = device
        self.num_pages = num_pages
        self.page_size = page_size
        self.ring = torch.arange(num_pages, dtype=torch.int32, device=device)
        self._head = 0
        self._tail = num_pages

    # -- reference API -------------------------------------------------------
    @property
    def available_size(self) -> int:
        return self._tail - self._head

    def allocate(self, needed_len: int) -> torch.Tensor:
        if needed_len < 0:
            raise ValueError("needed_len must be non-negative")
        if needed_len > self.available_size:
            raise NotImplementedError("CacheManager eviction is not implemented.")
        out = ops.slot_alloc(self.ring, self._head, needed_len)
        self._head += needed_len
        return out

    def _free(self, indices: torch.Tensor) -> None:
        n = int(indices.numel())
        if n == 0:
            return
        if self.available_size + n > self.num_pages:
            raise RuntimeError("CacheManager double free: more ids returned than the pool holds")
        ops.slot_free(self.ring, self._tail, indices)
        self._tail += n

    def allocate_paged(self, reqs: list[Req], page_table: torch.Tensor) -> None:
        for req in reqs:
            assert req.table_idx is not None
            extend_len = req.extend_len
            if extend_len == 0:
                continue
            page_table[req.table_idx, req.cached_len : req.device_len] = self.allocate(extend_len)

    # -- device-side allocation support -------------------------------------
    @property
    def head(self) -> int:
        return self._head

    @property
    def tail(self) -> int:
        return self._tail

    def advance_head(self, new_head: int) -> None:
        """Records ids the device took from the front of the ring."""
        if not self._head <= new_head <= self._tail:
            raise RuntimeError(f"device allocator head {new_head} outside [{self._head}, {self._tail}]")
        self._head = new_head

    def free_range(self, begin: int, count: int) -> None:
        """Returns ring entries [begin, begin + count) (ids allocated in that
        order) to the tail, like ``_free(torch.cat(allocated_pages))``."""
        if count == 0:
            return
        if not (0 <= begin and begin + count <= self._head):
            raise RuntimeError("free_range outside the allocated part of the ring")
        if self._tail - begin > self.num_pages:
            raise RuntimeError("free_range source already recycled")
        ops.slot_free_range(self.ring, begin, count, self._tail)
        self._tail += count
