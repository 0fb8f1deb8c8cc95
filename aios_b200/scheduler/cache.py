"""Free-slot FIFO of the paged KV pool (replaces aios/scheduler/cache.py:9-51).

The free list is kept twice, identically: as a device ring of ``num_pages``
int32 ids (read by the CandidateGroup step kernel, which allocates decode slots
on the device) and as a host list mirror. ``allocate(n)`` hands out the first n
free ids and ``_free`` appends at the tail, so ids come back in exactly the
reference's FIFO order (initially ``arange(num_pages)``). Allocation only moves
the head; frees write the returned ids to the ring's tail with one host-to-device
copy. After a device-side round the host advances its head by the count the
device reports and, knowing the ring order, knows every id the device took.

With ``page_size`` 1 an id is a token slot (the reference layout); with 16 an id
is a page of 16 consecutive token slots.

The ring may also live on the CPU (``device="cpu"``), as the reference's list can:
the same host logic then runs without a GPU (ids are written straight into the
ring), which is what the CPU tests of the allocator use. The CandidateGroup
runtime needs the CUDA ring.
"""

from __future__ import annotations

import torch

from ..core import Req


class CacheManager:
    def __init__(self, device: torch.device, num_pages: int, page_size: int = 1):
        device = torch.device(device)
        if device.type not in ("cuda", "cpu"):
            raise ValueError("CacheManager keeps its free list on a CUDA device (or the CPU)")
        if num_pages < 1:
            raise ValueError("num_pages must be positive")
        self.device = device
        self.num_pages = num_pages
        self.page_size = page_size
        self.ring = torch.arange(num_pages, dtype=torch.int32, device=device)
        self._host = list(range(num_pages))  # ring contents, index = logical position % num_pages
        self._head = 0
        self._tail = num_pages
        self._on_cuda = device.type == "cuda"
        if self._on_cuda:
            self._staging = torch.zeros(num_pages, dtype=torch.int32).pin_memory()
            self._stage_np = self._staging.numpy()
            self._stage_event = torch.cuda.Event()
        self._stage_busy = False

    # -- reference API -------------------------------------------------------
    @property
    def available_size(self) -> int:
        return self._tail - self._head

    def allocate(self, needed_len: int) -> torch.Tensor:
        """First `needed_len` free ids as a device tensor (reference API)."""
        ids = self.take(needed_len)
        return self._to_device(ids)

    def _free(self, indices) -> None:
        """Append ids (device tensor, host tensor or list) at the tail."""
        if isinstance(indices, torch.Tensor):
            ids = indices.to("cpu", torch.int64).tolist()
        else:
            ids = [int(i) for i in indices]
        self.give(ids)

    def allocate_paged(self, reqs: list[Req], page_table: torch.Tensor) -> None:
        for req in reqs:
            assert req.table_idx is not None
            extend_len = req.extend_len
            if extend_len == 0:
                continue
            page_table[req.table_idx, req.cached_len : req.device_len] = self.allocate(extend_len)

    # -- host-side allocation ----------------------------------------------------
    def take(self, n: int) -> list[int]:
        """First n free ids, as host ints (no device work)."""
        if n < 0:
            raise ValueError("needed_len must be non-negative")
        if n > self.available_size:
            raise NotImplementedError("CacheManager eviction is not implemented.")
        cap = self.num_pages
        out = [self._host[(self._head + i) % cap] for i in range(n)]
        self._head += n
        return out

    def give(self, ids: list[int]) -> None:
        """Append ids at the tail of both copies of the ring."""
        n = len(ids)
        if n == 0:
            return
        if self.available_size + n > self.num_pages:
            raise RuntimeError("CacheManager double free: more ids returned than the pool holds")
        cap = self.num_pages
        start = self._tail % cap
        for i, v in enumerate(ids):
            self._host[(start + i) % cap] = int(v)
        self._write_ring(start, ids)
        self._tail += n

    def _write_ring(self, start: int, ids: list[int]) -> None:
        n = len(ids)
        cap = self.num_pages
        first = min(n, cap - start)
        if not self._on_cuda:
            self.ring[start : start + first] = torch.tensor(ids[:first], dtype=torch.int32)
            if first < n:
                self.ring[: n - first] = torch.tensor(ids[first:], dtype=torch.int32)
            return
        if self._stage_busy:
            self._stage_event.synchronize()  # previous copy still reads the staging buffer
        self._stage_np[:n] = ids
        self.ring[start : start + first].copy_(self._staging[:first], non_blocking=True)
        if first < n:
            self.ring[: n - first].copy_(self._staging[first:n], non_blocking=True)
        self._stage_event.record()
        self._stage_busy = True

    def _to_device(self, ids: list[int]) -> torch.Tensor:
        if not self._on_cuda:
            return torch.tensor(ids, dtype=torch.int32)
        return torch.tensor(ids, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)

    # -- device-side allocation support -----------------------------------------
    @property
    def head(self) -> int:
        return self._head

    @property
    def tail(self) -> int:
        return self._tail

    def peek(self, begin: int, count: int) -> list[int]:
        """Ring entries [begin, begin + count) (ids handed out in that order)."""
        cap = self.num_pages
        return [self._host[(begin + i) % cap] for i in range(count)]

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
        self.give(self.peek(begin, count))
