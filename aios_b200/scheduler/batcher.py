"""Continuous batching for the generic ``LLM.generate`` path, on the same kernels
as the IME path. It keeps the reference's scheduling behaviour
(aios/scheduler/scheduler.py:19-176, driven by aios/llm/llm.py:98-175):
prefill first, varlen prefill batches of whole prompts, one decode token per
running request otherwise, page_size 1 KV slots claimed as batches are built and
returned the moment a request finishes. There is no prefix caching and no
chunked prefill.

Host-side state is plain Python: each request keeps its prompt, its generated
ids and the KV slots it holds, so a batch never gathers token ids on the device.
Admission keeps one running count of the KV slots the running requests may still
claim (prompt + max_tokens each, less what they already hold) and admits pending
requests in arrival order while a page-table row is free, the running set stays
under ``max_running``, the free slots cover the new request on top of every
claim, and the prefill token budget (if any) allows it; the first request of a
batch is always within the budget. The running set is a list in admission order.
Each batch stages its token ids, positions, page-table rows and new slots in one
pinned buffer, copies it to the device once, and writes its page-table entries
with one scatter.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..core import Batch, Req, SamplingParams
from .cache import CacheManager


@dataclass(eq=False)
class _Request:
    uid: int
    prompt: list[int]
    params: SamplingParams
    req: Req | None = None  # the batch-facing view, once admitted
    slots: list[int] = field(default_factory=list)  # KV slots held, position order
    generated: list[int] = field(default_factory=list)

    @property
    def claim(self) -> int:
        """KV slots this request may hold in total (as the reference reserves them)."""
        return len(self.prompt) + self.params.max_tokens


class ContinuousBatcher:
    def __init__(self, *, cache_manager: CacheManager, page_table: torch.Tensor, eos_token_id: int | None,
                 device: torch.device, max_running: int, attn_backend, prefill_token_budget: int | None = None):
        if max_running < 1 or max_running > page_table.shape[0]:
            raise ValueError("max_running must be in [1, page-table rows]")
        self.cache = cache_manager
        self.page_table = page_table
        self.eos = eos_token_id
        self.device = device
        self.max_running = max_running
        self.attn_backend = attn_backend
        self.budget = prefill_token_budget
        self._free_rows = sorted(range(max_running), reverse=True)  # pop() takes the lowest row
        self._pending: list[_Request] = []
        self._running: list[_Request] = []
        self._done: list[_Request] = []
        self._live: dict[int, _Request] = {}  # admitted and not finished, by uid
        self._outstanding = 0  # KV slots the running requests may still claim
        self._uid = 0

    # ---- requests ------------------------------------------------------------
    def add_request(self, input_ids: torch.Tensor | list[int], sampling_params: SamplingParams) -> int:
        ids = input_ids.tolist() if isinstance(input_ids, torch.Tensor) else [int(t) for t in input_ids]
        if not ids:
            raise ValueError("a request needs at least one prompt token")
        uid = self._uid
        self._uid += 1
        self._pending.append(_Request(uid=uid, prompt=ids, params=sampling_params))
        return uid

    @property
    def has_work(self) -> bool:
        return bool(self._pending or self._running)

    # ---- batch construction --------------------------------------------------
    def _admit(self) -> list[_Request]:
        free = self.cache.available_size - self._outstanding
        rows = len(self._free_rows)
        room = self.max_running - len(self._running)
        tokens, chosen = 0, []
        for r in self._pending:
            n = len(r.prompt)
            if chosen and self.budget is not None and tokens + n > self.budget:
                break
            if len(chosen) >= min(rows, room) or r.claim > free:
                break
            chosen.append(r)
            free -= r.claim
            tokens += n
            if self.budget is not None and tokens >= self.budget:
                break
        del self._pending[: len(chosen)]
        return chosen

    def next_batch(self) -> Batch | None:
        """The next forward: a prefill of newly admitted requests when any can be
        admitted, else one decode token of every running request; None when
        nothing can run (pending requests that do not fit the free KV slots)."""
        admitted = self._admit()
        if admitted:
            for r in admitted:
                r.req = Req(input_ids=torch.tensor(r.prompt, dtype=torch.long), cached_len=0,
                            output_len=r.params.max_tokens, uid=r.uid, sampling_params=r.params,
                            table_idx=self._free_rows.pop())
                self._outstanding += r.claim
                self._live[r.uid] = r
            return self._stage(admitted, "prefill")
        if self._running:
            return self._stage(list(self._running), "decode")
        return None

    def _stage(self, group: list[_Request], phase: str) -> Batch:
        ids, pos, rows, counts = [], [], [], []
        for r in group:
            req = r.req
            new = range(req.cached_len, req.device_len)
            ids += r.prompt if phase == "prefill" else [r.generated[-1]]
            pos += new
            rows += [req.table_idx] * len(new)
            counts.append(len(new))
        slots = self.cache.take(len(ids))  # FIFO order, request by request
        at = 0
        for r, n in zip(group, counts):
            r.slots += slots[at : at + n]
            at += n
        self._outstanding -= len(ids)
        n = len(ids)
        host = torch.tensor(ids + pos + rows + slots, dtype=torch.int32)
        if self.device.type == "cuda":
            host = host.pin_memory()
        dev = host.to(self.device, non_blocking=True)
        b = Batch(reqs=[r.req for r in group], phase=phase)
        b.input_ids = dev[:n].long()
        b.positions = dev[n : 2 * n]
        row_t, slot_t = dev[2 * n : 3 * n], dev[3 * n :]
        b.out_loc = slot_t
        self.page_table[row_t.long(), b.positions.long()] = slot_t
        self.attn_backend.prepare_metadata(b)
        return b

    # ---- results ---------------------------------------------------------------
    def commit(self, batch: Batch, next_tokens: torch.Tensor) -> None:
        """Appends each request's sampled token; finished requests return their KV
        slots and table row at once, new prefills join the running set."""
        group = [self._live[req.uid] for req in batch.reqs]
        finished = set()
        for r, tok in zip(group, next_tokens.view(-1).tolist()):
            r.req.complete_one()
            r.generated.append(tok)
            stop = (not r.params.ignore_eos and self.eos is not None and tok == self.eos) or not r.req.can_decode
            if stop:
                finished.add(r.uid)
                self._release(r)
        if batch.is_prefill:
            self._running += [r for r in group if r.uid not in finished]
        else:
            self._running = [r for r in self._running if r.uid not in finished]

    def _release(self, r: _Request) -> None:
        self._outstanding -= r.claim - len(r.slots)
        self.cache.give(r.slots)
        r.slots = []
        self._free_rows.append(r.req.table_idx)
        self._free_rows.sort(reverse=True)
        del self._live[r.uid]
        self._done.append(r)

    def results(self, tokenizer) -> list[dict]:
        out = [{"uid": r.uid, "token_ids": r.generated,
                "text": tokenizer.decode(r.generated, skip_special_tokens=True)} for r in self._done]
        return sorted(out, key=lambda d: d["uid"])

    def describe(self, batch: Batch | None = None) -> str:
        return (f"batch={batch.phase if batch else None}:{[r.uid for r in batch.reqs] if batch else []} "
                f"pending={[r.uid for r in self._pending]} running={[r.uid for r in self._running]} "
                f"done={[r.uid for r in self._done]} free_slots={self.cache.available_size} "
                f"claimed={self._outstanding}")
