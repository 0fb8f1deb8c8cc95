"""End-to-end CandidateGroup behaviour on the GPU (mirrors the reference's
tests/test_ime_gpu.py on seeded synthetic weights instead of a checkpoint)."""

from __future__ import annotations

import threading
import time

import pytest
import torch

from aios_b200 import ImeCompletionEngine, ImeGenerationConfig, LLM
from aios_b200.models.shapes import S10

pytestmark = pytest.mark.gpu


def _prefix(llm, n: int, seed: int) -> str:
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(10, llm.config.vocab_size, (n,), generator=g).tolist()
    return llm.tokenizer.text_for(ids)


@pytest.fixture(scope="module", params=[1, 16], ids=["page1", "page16"])
def engine(request) -> ImeCompletionEngine:
    page_size = request.param
    llm = LLM(config=S10, seed=0, page_size=page_size, num_pages=4096 if page_size == 1 else 256)
    eng = ImeCompletionEngine(llm)
    eng.complete(_prefix(llm, 4, 1), ImeGenerationConfig(seed=1))
    return eng


def test_candidate_group_recycles_branch_pages(engine) -> None:
    llm = engine.llm
    engine.reset_prefix_cache()
    prefix = _prefix(llm, 12, 7)
    cfg = ImeGenerationConfig(seed=7, temperature=0.8, max_sampling_attempts=24)
    result = engine.complete(prefix, cfg)
    assert 8 <= result.sampling_attempts <= 24
    assert result.prefix_tokens == 13
    assert len(result.raw_candidates) == result.sampling_attempts
    assert result.gpu_latency_ms > 0
    # only the persistent prefix stays allocated
    used = llm.num_pages - llm.cache_manager.available_size
    assert used == -(-result.prefix_tokens // llm.cache_manager.page_size)


def test_incremental_prefix_reuses_token_lcp(engine) -> None:
    llm = engine.llm
    engine.reset_prefix_cache()
    base = _prefix(llm, 10, 11)
    cfg = ImeGenerationConfig(seed=11, max_sampling_attempts=8)
    first = engine.complete(base[:6], cfg)
    extended = engine.complete(base, cfg)
    repeated = engine.complete(base, cfg)
    assert first.reused_prefix_tokens == 0
    assert extended.reused_prefix_tokens == 7
    assert repeated.reused_prefix_tokens == repeated.prefix_tokens
    # identical prefix -> identical candidates (deterministic stateless streams)
    assert [c.text for c in extended.raw_candidates] == [c.text for c in repeated.raw_candidates]


def test_long_prefix_prefill_then_short_extension(engine) -> None:
    """A 100-token prefix prefills more than 64 new tokens (norm/RoPE/store and
    attention as two launches); extending it by a few tokens prefills over 101
    cached keys on the one-launch path, whose key chunks mix cached and new keys.
    Any device-side range report would raise here."""
    llm = engine.llm
    engine.reset_prefix_cache()
    text = _prefix(llm, 104, 23)
    cfg = ImeGenerationConfig(seed=23, max_sampling_attempts=8)
    long_result = engine.complete(text[:100], cfg)
    assert long_result.prefix_tokens == 101 and long_result.reused_prefix_tokens == 0
    extended = engine.complete(text, cfg)
    assert extended.prefix_tokens == 105 and extended.reused_prefix_tokens == 101
    assert len(extended.raw_candidates) == extended.sampling_attempts


def test_latest_generation_cancels_old_group_and_frees_pages(engine) -> None:
    llm = engine.llm
    box: dict[str, object] = {}
    old = engine.new_generation()
    cfg = ImeGenerationConfig(max_new_tokens=64, min_new_tokens=64, max_candidate_chars=100, seed=17,
                              max_sampling_attempts=8)

    def run_old() -> None:
        box["result"] = engine.complete(_prefix(llm, 30, 17), cfg, old)

    worker = threading.Thread(target=run_old)
    worker.start()
    time.sleep(0.003)
    new = engine.new_generation()
    worker.join(timeout=30)
    assert not worker.is_alive()
    current = engine.complete(_prefix(llm, 5, 19), ImeGenerationConfig(seed=19), new)
    assert not current.cancelled
    engine.reset_prefix_cache()
    assert llm.cache_manager.available_size == llm.num_pages
    assert isinstance(box["result"].cancelled, bool)


def test_greedy_rows_are_identical(engine) -> None:
    """Greedy (top_k=1, top_p=1): all 8 rows see the same logits and must agree."""
    llm = engine.llm
    engine.reset_prefix_cache()
    cfg = ImeGenerationConfig(seed=3, top_k=1, top_p=1.0, temperature=1.0, max_sampling_attempts=8, min_new_tokens=0)
    result = engine.complete(_prefix(llm, 8, 3), cfg)
    texts = {c.text for c in result.raw_candidates}
    assert len(texts) == 1


def test_keystroke_with_a_top_k_beyond_the_top_k_buffer(engine) -> None:
    """top_k 4096 (any top_k >= 1 the reference accepts, aios/ime.py:87): the
    step sorts whole rows; the round completes with valid candidates, and the
    usual 2048-or-less setting still runs its own step graph."""
    llm = engine.llm
    engine.reset_prefix_cache()
    prefix = _prefix(llm, 12, 31)
    wide = engine.complete(prefix, ImeGenerationConfig(seed=31, top_k=4096, top_p=0.9, max_sampling_attempts=8))
    assert wide.sampling_attempts == 8 and len(wide.raw_candidates) == 8
    assert all(0 < c.token_count <= 12 for c in wide.raw_candidates)
    narrow = engine.complete(prefix, ImeGenerationConfig(seed=31, top_k=50, top_p=0.9, max_sampling_attempts=8))
    assert narrow.sampling_attempts == 8
    keys = set(engine._runtime._graphs)
    assert {k[:2] for k in keys} >= {(8, True), (8, False)}
