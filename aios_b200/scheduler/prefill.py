"""Admission of pending requests into one varlen prefill batch
(aios/scheduler/prefill.py:1-100).

A request is admitted while a table row is free, the running set stays under
`max_running`, and the free KV slots cover its prompt and output plus what the
running set and the requests admitted in this batch may still claim. A prefill
token budget (if given) caps the prompt tokens of one batch, with at least one
request always admitted.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import TYPE_CHECKING, List

import torch

from ..core import Batch, Req
from .common import PendingReq

if TYPE_CHECKING:
    from .cache import CacheManager
    from .decode import DecodeManager
    from .table import TableManager


@dataclass
class PrefillManager:
    cache_manager: "CacheManager"
    table_manager: "TableManager"
    decode_manager: "DecodeManager"
    pending_list: List[PendingReq] = field(default_factory=list)

    def add_one_req(self, pending: PendingReq) -> None:
        self.pending_list.append(pending)

    @property
    def runnable(self) -> bool:
        return bool(self.pending_list)

    def _can_admit(self, pending: PendingReq, max_running: int, scheduled: int, scheduled_reserved: int) -> bool:
        if self.table_manager.available_size - scheduled <= 0:
            return False
        if len(self.decode_manager.running_reqs) + scheduled >= max_running:
            return False
        needed = pending.input_len + pending.output_len
        reserved = self.decode_manager.inflight_tokens + scheduled_reserved
        return needed + reserved <= self.cache_manager.available_size

    def schedule_next_batch(self, max_running: int, max_prefill_tokens: int | None = None) -> Batch | None:
        if not self.pending_list:
            return None
        budget = max_prefill_tokens if max_prefill_tokens is not None else float("inf")
        selected: List[PendingReq] = []
        tokens = 0
        reserved = 0
        for pending in self.pending_list:
            if selected and tokens + pending.input_len > budget:
                break
            if not self._can_admit(pending, max_running, len(selected), reserved):
                break
            selected.append(pending)
            tokens += pending.input_len
            reserved += pending.input_len + pending.output_len
            if tokens >= budget:
                break
        if not selected:
            return None
        self.pending_list = self.pending_list[len(selected):]
        reqs: List[Req] = []
        for pending in selected:
            row = self.table_manager.allocate()
            self.table_manager.token_pool[row, : pending.input_len] = pending.input_ids.to(torch.int32)
            reqs.append(Req(input_ids=pending.input_ids, cached_len=0, output_len=pending.output_len, uid=pending.uid,
                            sampling_params=pending.sampling_params, table_idx=row))
        return Batch(reqs=reqs, phase="prefill")
