"""Request rows of the generic ``LLM.generate`` path (aios/scheduler/table.py:1-22).

Each running request owns one row of the page table (its KV slot per position)
and the same row of a device token pool (its prompt and generated ids, from
which decode batches gather their inputs). Rows come from the end of the free
list and go back to it when a request finishes, as in the reference.
"""

from __future__ import annotations

import torch


class TableManager:
    def __init__(self, max_running_reqs: int, page_table: torch.Tensor) -> None:
        self._free_slots = list(range(max_running_reqs))
        self.page_table = page_table
        self.token_pool = torch.zeros_like(page_table, dtype=torch.int32)

    @property
    def available_size(self) -> int:
        return len(self._free_slots)

    def allocate(self) -> int:
        return self._free_slots.pop()

    def free(self, slot: int) -> None:
        self._free_slots.append(slot)
