"""Continuous-batching scheduler of the generic ``LLM.generate`` path
(aios/scheduler/scheduler.py:19-176).

Prefill first: each iteration admits a varlen prefill batch of pending requests
when it can, otherwise decodes one token for every running request. KV slots
(page_size 1) are taken from the FIFO when a batch is prepared and returned the
moment a request finishes, so a pending request can use them in the next
iteration. No prefix caching and no chunked prefill, as in the reference.
"""

from __future__ import annotations

from typing import List

import torch

from ..attention import BaseAttentionBackend
from ..core import Batch, Req, SamplingParams
from .cache import CacheManager
from .common import PendingReq
from .decode import DecodeManager
from .prefill import PrefillManager
from .table import TableManager


class Scheduler:
    def __init__(self, table_manager: TableManager, cache_manager: CacheManager, eos_token_id: int,
                 device: torch.device, max_running_reqs: int, attn_backend: BaseAttentionBackend,
                 prefill_token_budget: int | None = None) -> None:
        self.table_manager = table_manager
        self.cache_manager = cache_manager
        self.eos_token_id = eos_token_id
        self.device = device
        self.max_running = max_running_reqs
        self.attn_backend = attn_backend
        self.prefill_token_budget = prefill_token_budget
        self.decode_manager = DecodeManager(page_size=1)
        self.prefill_manager = PrefillManager(cache_manager=cache_manager, table_manager=table_manager,
                                              decode_manager=self.decode_manager)
        self.finished: List[Req] = []
        self._next_uid = 0

    def add_request(self, input_ids: torch.Tensor, sampling_params: SamplingParams) -> int:
        uid = self._next_uid
        self._next_uid += 1
        self.prefill_manager.add_one_req(PendingReq(uid=uid, input_ids=input_ids, sampling_params=sampling_params))
        return uid

    def schedule_next_batch(self) -> Batch | None:
        batch = (self.prefill_manager.schedule_next_batch(self.max_running, self.prefill_token_budget)
                 or self.decode_manager.schedule_next_batch())
        return self._prepare_batch(batch) if batch else None

    def _prepare_batch(self, batch: Batch) -> Batch:
        """KV slots for the new tokens, then positions, input ids and slots of every
        token of the batch in one host-to-device copy, then the attention metadata."""
        table = self.table_manager.page_table
        self.cache_manager.allocate_paged(batch.reqs, table)
        rows, positions = [], []
        for req in batch.reqs:
            rows += [req.table_idx] * req.extend_len
            positions += range(req.cached_len, req.device_len)
        staged = torch.tensor(rows + positions, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True)
        row_idx, pos_idx = staged[: len(rows)], staged[len(rows):]
        batch.positions = pos_idx.to(torch.int32)
        batch.input_ids = self.table_manager.token_pool[row_idx, pos_idx].long()
        batch.out_loc = table[row_idx, pos_idx]
        self.attn_backend.prepare_metadata(batch)
        return batch

    def process_batch_output(self, batch: Batch, next_tokens: torch.Tensor) -> None:
        tokens = next_tokens.view(-1).tolist()
        for req, tok in zip(batch.reqs, tokens):
            if self._advance(req, tok):
                if batch.is_decode:
                    self.decode_manager.remove_req(req)
                self._free_req_resources(req)
                self.finished.append(req)
        if batch.is_prefill:
            done = set(map(id, self.finished))
            self.decode_manager.filter_reqs([req for req in batch.reqs if id(req) not in done])

    def debug_state(self, batch: Batch | None = None) -> str:
        return (f"Batch={batch} Pending={self.prefill_manager.pending_list} "
                f"Running={self.decode_manager.running_reqs} Finished={self.finished}")

    def _advance(self, req: Req, tok: int) -> bool:
        req.complete_one()
        self.table_manager.token_pool[req.table_idx, req.device_len - 1] = tok
        req.generated.append(tok)
        hit_eos = (not req.sampling_params.ignore_eos) and tok == self.eos_token_id
        return hit_eos or not req.can_decode

    def _free_req_resources(self, req: Req) -> None:
        used = self.table_manager.page_table[req.table_idx, : req.cached_len]
        self.table_manager.free(req.table_idx)
        self.cache_manager._free(used)

    @property
    def has_work(self) -> bool:
        return self.prefill_manager.runnable or self.decode_manager.runnable

    def collect_results(self, tokenizer) -> list[dict]:
        results = [{"uid": req.uid, "token_ids": req.generated,
                    "text": tokenizer.decode(req.generated, skip_special_tokens=True)} for req in self.finished]
        results.sort(key=lambda r: r["uid"])
        return results
