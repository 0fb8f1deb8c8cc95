"""The generic continuous-batching ``LLM.generate`` (aios/llm/llm.py:98-175) on the
B200 kernels, against the CPU oracle.

Greedy requests of different prompt and output lengths run with fewer running
slots than requests and a prefill token budget, so admission, varlen prefill,
decode batches of changing size and slot recycling are all exercised. The oracle
replays every request teacher-forced on the GPU's tokens: each GPU token is the
oracle's argmax, except at bf16 near-ties (top-1/top-2 gap under 2e-2), as in
the keystroke parity tests.
"""

from __future__ import annotations

import dataclasses

import pytest
import torch

from aios_b200 import LLM
from aios_b200.core import SamplingParams
from aios_b200.models import shapes
from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM
from aios_b200.models.weight import synthetic_state_dict
from oracle.model import OracleModel, Request

pytestmark = pytest.mark.gpu

GREEDY_MARGIN = 2e-2


def _oracle(cfg, num_slots: int) -> OracleModel:
    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    state = {k: v.to(torch.bfloat16) for k, v in synthetic_state_dict(meta, seed=0).items()}
    return OracleModel(cfg, state, dtype=torch.bfloat16, num_slots=num_slots, mixer="fused")


def _replay(oracle: OracleModel, prompt: list[int], generated: list[int], first_slot: int) -> int:
    """Teacher-forced oracle decode of one request; returns the near-tie flips."""
    n = len(prompt)
    slots = list(range(first_slot, first_slot + n + len(generated)))
    logits = oracle.forward([Request(ids=prompt, positions=list(range(n)), new_slots=slots[:n], key_slots=slots[:n])])
    flips = 0
    for step, tok in enumerate(generated):
        row = logits[0].float()
        top2 = torch.topk(row, 2)
        if int(top2.indices[0]) != tok:
            assert float(top2.values[0] - top2.values[1]) < GREEDY_MARGIN, (step, tok, int(top2.indices[0]))
            flips += 1
        if step + 1 < len(generated):
            pos = n + step
            logits = oracle.forward([Request(ids=[tok], positions=[pos], new_slots=[slots[pos]],
                                             key_slots=slots[: pos + 1])])
    return flips


@pytest.mark.parametrize("cfg", [dataclasses.replace(shapes.S10, num_layers=2),
                                 dataclasses.replace(shapes.S21, num_layers=4, attnres_num_blocks=2)],
                         ids=["s10_l2", "s21_l4"])
def test_generate_greedy_matches_oracle(cfg) -> None:
    llm = LLM(config=cfg, seed=0, page_size=1, num_pages=1024)
    g = torch.Generator().manual_seed(3)
    prompts = [[1] + torch.randint(10, cfg.vocab_size, (n,), generator=g).tolist() for n in (3, 17, 8, 11, 5)]
    params = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True) for m in (6, 4, 9, 3, 7)]
    results = llm.generate(prompts, params, max_running_reqs=3, prefill_token_budget=24)
    assert [r["uid"] for r in results] == list(range(len(prompts)))
    assert [len(r["token_ids"]) for r in results] == [p.max_tokens for p in params]
    # every KV slot went back to the free list
    assert llm.cache_manager.available_size == llm.num_pages
    oracle = _oracle(cfg, 1024)
    flips = sum(_replay(oracle, p, r["token_ids"], 0) for p, r in zip(prompts, results))
    assert flips <= 2


def test_generate_sampled_and_mixed_params() -> None:
    cfg = dataclasses.replace(shapes.S10, num_layers=2)
    llm = LLM(config=cfg, seed=0, page_size=1, num_pages=256)
    prompts = ["今天天气", "你好", "我们"]
    params = [SamplingParams(temperature=0.8, top_k=20, top_p=0.9, max_tokens=5, ignore_eos=True),
              SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True),
              SamplingParams(temperature=1.0, top_k=50, top_p=0.8, max_tokens=6, ignore_eos=True)]
    results = llm.generate(prompts, params, prompt_mode="raw")
    assert [len(r["token_ids"]) for r in results] == [5, 4, 6]
    assert all(0 <= t < cfg.vocab_size for r in results for t in r["token_ids"])
    assert all(r["text"] == llm.tokenizer.decode(r["token_ids"]) for r in results)
    assert llm.cache_manager.available_size == llm.num_pages
    # a top-p-only sampler (top_k 0, aios/engine/sample.py:131-132) sorts the whole vocabulary
    topp = llm.generate(prompts[:1], SamplingParams(temperature=1.0, top_p=0.8, max_tokens=2), prompt_mode="raw")
    assert len(topp[0]["token_ids"]) >= 1 and all(0 <= t < cfg.vocab_size for t in topp[0]["token_ids"])
    assert llm.cache_manager.available_size == llm.num_pages
    with pytest.raises(ValueError, match="page_size 1"):
        LLM(config=cfg, seed=0, page_size=16, num_pages=16).generate(prompts, params, prompt_mode="raw")
