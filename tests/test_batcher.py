"""The continuous batcher of ``LLM.generate`` on the CPU: its host logic only
(admission, batch staging, KV slot and row accounting, results), with a
stand-in forward that emits a fixed token per request and step.

Checked against the reference's scheduling rules (aios/scheduler/prefill.py,
decode.py, scheduler.py): prefill before decode; a request is admitted while a
table row is free, the running set is under its cap and the free KV slots cover
its prompt + max_tokens on top of every running claim; the prefill token budget
caps a batch, whose first request is always admitted; one decode token per
running request; a finished request returns its slots and row at once."""

from __future__ import annotations

import torch

from aios_b200.core import SamplingParams
from aios_b200.scheduler import CacheManager, ContinuousBatcher

EOS = 2


class _NoMetadata:
    def __init__(self):
        self.batches = []

    def prepare_metadata(self, batch):
        self.batches.append((batch.phase, [r.uid for r in batch.reqs]))


def _token(uid: int, step: int, eos_at: dict) -> int:
    return EOS if eos_at.get(uid) == step else 100 + 10 * uid + step


def _run(prompts, params, *, pages=64, max_running=3, budget=None, eos_at=None):
    eos_at = eos_at or {}
    cm = CacheManager(torch.device("cpu"), pages)
    table = torch.zeros((max_running, 64), dtype=torch.int32)
    backend = _NoMetadata()
    b = ContinuousBatcher(cache_manager=cm, page_table=table, eos_token_id=EOS, device=torch.device("cpu"),
                          max_running=max_running, attn_backend=backend, prefill_token_budget=budget)
    for p, sp in zip(prompts, params):
        b.add_request(p, sp)
    steps: dict[int, int] = {}
    trace = []
    while b.has_work:
        batch = b.next_batch()
        assert batch is not None
        n_tokens = batch.input_ids.numel()
        assert batch.positions.numel() == batch.out_loc.numel() == n_tokens
        # every staged slot is written into the request's page-table row at its position
        at = 0
        for req in batch.reqs:
            n = req.extend_len
            rows = table[req.table_idx, req.cached_len : req.device_len]
            assert rows.tolist() == batch.out_loc[at : at + n].tolist()
            at += n
        running = len(b._running)
        assert running <= max_running
        trace.append((batch.phase, [r.uid for r in batch.reqs], n_tokens, cm.available_size))
        out = []
        for req in batch.reqs:
            s = steps.get(req.uid, 0)
            out.append(_token(req.uid, s, eos_at))
            steps[req.uid] = s + 1
        b.commit(batch, torch.tensor(out))
    return b, cm, trace


def test_prefill_first_and_running_cap() -> None:
    prompts = [[1, 10, 11], [1, 12], [1, 13, 14, 15], [1, 16]]
    params = [SamplingParams(max_tokens=m, ignore_eos=True) for m in (3, 2, 4, 1)]
    b, cm, trace = _run(prompts, params, max_running=2)
    # the first two requests fill the two rows; the others wait for a finish
    assert trace[0][:2] == ("prefill", [0, 1])
    assert trace[1][:2] == ("decode", [0, 1])
    phases = [t[0] for t in trace]
    assert phases.count("prefill") == 3  # [0, 1], then [2] and [3] as rows free up
    res = b.results(_Tok())
    assert [r["uid"] for r in res] == [0, 1, 2, 3]
    assert [len(r["token_ids"]) for r in res] == [3, 2, 4, 1]
    assert res[0]["token_ids"] == [100, 101, 102]
    assert cm.available_size == 64  # every slot returned


def test_prefill_budget_and_first_request() -> None:
    prompts = [[1] * 9, [1] * 5, [1] * 5, [1] * 2]
    params = [SamplingParams(max_tokens=2, ignore_eos=True)] * 4
    b, cm, trace = _run(prompts, params, max_running=4, budget=8)
    prefills = [t for t in trace if t[0] == "prefill"]
    # a 9-token prompt exceeds the 8-token budget but is admitted alone; then 5
    # (5 + 5 > 8 stops the batch), then 5 + 2
    assert [p[1] for p in prefills] == [[0], [1], [2, 3]]
    assert [p[2] for p in prefills] == [9, 5, 7]
    assert cm.available_size == 64


def test_kv_capacity_admission_and_eos() -> None:
    # 20 slots: each request claims prompt + max_tokens = 10, so two fit at a time
    prompts = [[1, 20, 21, 22]] * 3
    params = [SamplingParams(max_tokens=6)] * 3
    b, cm, trace = _run(prompts, params, pages=20, max_running=3, eos_at={0: 1})
    assert trace[0][:2] == ("prefill", [0, 1])
    # request 0 stops on EOS at its second token; its slots admit request 2
    res = b.results(_Tok())
    assert res[0]["token_ids"] == [100, EOS]
    assert [len(r["token_ids"]) for r in res] == [2, 6, 6]
    later = [t for t in trace if t[0] == "prefill"][1]
    assert later[1] == [2]
    assert cm.available_size == 20


def test_slots_come_out_in_fifo_order() -> None:
    prompts = [[1, 30], [1, 31, 32]]
    params = [SamplingParams(max_tokens=2, ignore_eos=True)] * 2
    cm = CacheManager(torch.device("cpu"), 16)
    table = torch.zeros((2, 16), dtype=torch.int32)
    b = ContinuousBatcher(cache_manager=cm, page_table=table, eos_token_id=EOS, device=torch.device("cpu"),
                          max_running=2, attn_backend=_NoMetadata())
    for p, sp in zip(prompts, params):
        b.add_request(p, sp)
    batch = b.next_batch()
    assert batch.out_loc.tolist() == [0, 1, 2, 3, 4]  # request by request, positions in order
    assert batch.input_ids.tolist() == [1, 30, 1, 31, 32]
    assert batch.positions.tolist() == [0, 1, 0, 1, 2]
    b.commit(batch, torch.tensor([7, 8]))
    batch = b.next_batch()
    assert batch.phase == "decode" and batch.input_ids.tolist() == [7, 8]
    assert batch.positions.tolist() == [2, 3] and batch.out_loc.tolist() == [5, 6]


class _Tok:
    def decode(self, ids, skip_special_tokens=True):
        return " ".join(map(str, ids))
