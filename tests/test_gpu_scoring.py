"""score_candidates (aios/ime.py:642-889) on the GPU against the CPU oracle.

Each candidate is teacher-forced on the oracle as one fresh sequence [BOS, prefix,
candidate]; the raw log-probability of every candidate token is summed and
averaged. The GPU engine's stable mode (one varlen prefill with all logits) and
shared-decode mode (prefix prefill + lock-step teacher-forced decode) must agree
per candidate within the bf16 log-probability bound of the keystroke parity
tests, and rank the candidates the same wherever their scores are further apart
than that bound.
"""

from __future__ import annotations

import dataclasses
import math

import pytest
import torch

from aios_b200 import ImeCompletionEngine, LLM
from aios_b200.models import shapes
from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM
from aios_b200.models.weight import synthetic_state_dict
from oracle.model import OracleModel, Request

pytestmark = pytest.mark.gpu

LOGPROB_TOL = 2e-2


def _oracle_scores(oracle: OracleModel, prefix_ids: list[int], cands: list[list[int]]) -> list[tuple[float, float]]:
    out = []
    for ids in cands:
        seq = [*prefix_ids, *ids]
        n = len(seq)
        logits = oracle.forward([Request(ids=seq, positions=list(range(n)), new_slots=list(range(n)),
                                         key_slots=list(range(n)))], all_logits=True)
        lp = torch.log_softmax(logits.float(), -1)
        vals = [float(lp[len(prefix_ids) - 1 + j, t]) for j, t in enumerate(ids)]
        out.append((sum(vals), sum(vals) / len(vals)))
    return out


def _bound(oracle_logits_scale: float) -> float:
    ulp = 2.0 ** (math.floor(math.log2(max(oracle_logits_scale, 1e-30))) - 7)
    return max(LOGPROB_TOL, 3 * ulp)


@pytest.fixture(scope="module")
def models():
    cfg = dataclasses.replace(shapes.S10, num_layers=2)
    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    state = {k: v.to(torch.bfloat16) for k, v in synthetic_state_dict(meta, seed=0).items()}
    oracle = OracleModel(cfg, state, dtype=torch.bfloat16, num_slots=256, mixer="fused")
    return cfg, oracle


@pytest.mark.parametrize("mode,page_size,num_pages", [("stable", 1, 1024), ("stable", 16, 128),
                                                       ("shared_decode", 1, 1024)])
def test_score_candidates_matches_oracle(models, mode: str, page_size: int, num_pages: int) -> None:
    cfg, oracle = models
    llm = LLM(config=cfg, seed=0, page_size=page_size, num_pages=num_pages)
    engine = ImeCompletionEngine(llm)
    tok = llm.tokenizer
    g = torch.Generator().manual_seed(3)
    prefix_ids = torch.randint(10, cfg.vocab_size, (9,), generator=g).tolist()
    cands = [torch.randint(10, cfg.vocab_size, (n,), generator=g).tolist() for n in (1, 3, 5, 2, 4)]
    prefix = tok.text_for(prefix_ids)
    texts = [tok.text_for(ids) for ids in cands]
    free_before = llm.cache_manager.tail - llm.cache_manager.head
    result = engine.score_candidates(prefix, texts, mode=mode)
    torch.cuda.synchronize()
    expected = _oracle_scores(oracle, [tok.bos_token_id, *prefix_ids], cands)
    by_text = {c.text: c for c in result.candidates}
    assert len(result.candidates) == len(texts)
    bound = _bound(20.0)  # |logits| of the random-init model stay below 20
    for text, ids, (esum, eavg) in zip(texts, cands, expected):
        got = by_text[text]
        assert got.token_count == len(ids)
        assert abs(got.average_logprob - eavg) < bound, (mode, text, got.average_logprob, eavg)
        assert abs(got.sum_logprob - esum) < bound * len(ids), (mode, text, got.sum_logprob, esum)
    # ranking: descending average, consistent with the oracle where clearly separated
    avgs = [c.average_logprob for c in result.candidates]
    assert avgs == sorted(avgs, reverse=True)
    exp_avg = {t: e[1] for t, e in zip(texts, expected)}
    order = [c.text for c in result.candidates]
    for i in range(len(order)):
        for j in range(i + 1, len(order)):
            if exp_avg[order[j]] - exp_avg[order[i]] > 2 * bound:
                raise AssertionError(f"{mode}: {order[j]!r} should rank above {order[i]!r}")
    # every page taken for the candidates went back to the pool; shared-decode
    # keeps the prefix ([BOS] + prefix) cached for the next keystroke
    cm = llm.cache_manager
    kept = 0 if mode == "stable" else engine._pages_for(len(prefix_ids) + 1)
    assert cm.tail - cm.head == free_before - kept


def test_score_candidates_errors(models) -> None:
    cfg, _ = models
    llm = LLM(config=cfg, seed=0, page_size=16, num_pages=128)
    engine = ImeCompletionEngine(llm)
    with pytest.raises(ValueError, match="must not be empty"):
        engine.score_candidates("一", [])
    with pytest.raises(ValueError, match="Unsupported scoring mode"):
        engine.score_candidates("一", ["二"], mode="bogus")
    with pytest.raises(ValueError, match="page_size=1"):
        engine.score_candidates("一", ["二"], mode="shared_decode")
