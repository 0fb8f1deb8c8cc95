"""CPU tests of the host-side engine logic: the same known answers the
reference pins in tests/test_ime.py and tests/test_ime_attnres.py, run against
aios_b200 (candidate keys, terminal truncation, filters, MMR, LCP, config
validation, pool statistics, adaptive refill, AttnRes config gates and
checkpoint names)."""

from __future__ import annotations

import pytest
import torch

from aios_b200 import (
    ImeGenerationConfig,
    adaptive_refill_attempts,
    candidate_pool_stats,
    token_longest_common_prefix,
    truncate_at_terminal,
)
from aios_b200.ime import ImeCandidate, candidate_key, invalid_reasons, ngram_similarity, select_top_candidates
from aios_b200.models.config import ModelConfig


def candidate(text: str, score: float) -> ImeCandidate:
    return ImeCandidate(text=text, token_count=3, average_logprob=score, base_score=score, selection_score=score,
                        stop_reason="eos", invalid_reasons=())


def invalid_candidate(text: str, reason: str = "unfinished_fragment") -> ImeCandidate:
    return ImeCandidate(text=text, token_count=2, average_logprob=-0.1, base_score=float("-inf"),
                        selection_score=float("-inf"), stop_reason="max_new_tokens", invalid_reasons=(reason,))


def test_candidate_key_collapses_display_punctuation() -> None:
    assert candidate_key(" 我晚点回复。 ") == candidate_key("我晚点回复")


def test_decoded_terminal_recovers_first_complete_sentence() -> None:
    text, stopped = truncate_at_terminal("我马上处理好。后面的句子不应显示")
    assert stopped and text == "我马上处理好。"
    phrase, stopped = truncate_at_terminal("我先确认一下，再回复你")
    assert not stopped and phrase == "我先确认一下，再回复你"


def test_invalid_reasons_reject_empty_assistant_and_repeat() -> None:
    config = ImeGenerationConfig()
    assert invalid_reasons("", config) == ("empty",)
    assert "assistant_template" in invalid_reasons("作为一个AI，我建议", config)
    assert "repeated_ngram" in invalid_reasons("好的好的好的", config)
    assert "unfinished_fragment" in invalid_reasons("我晚点再", config)
    assert "boundary_repeat" in invalid_reasons("好好休息", config, prefix="你好")
    assert "too_short" in invalid_reasons("好", config)
    assert "too_long" in invalid_reasons("好" * 40, ImeGenerationConfig(max_candidate_chars=32))


def test_boundary_repeat_allows_natural_word_boundary() -> None:
    assert "boundary_repeat" not in invalid_reasons("天气有点热，我先喝点水", ImeGenerationConfig(), prefix="今天")


def test_mmr_selection_keeps_quality_and_diversity() -> None:
    items = [
        candidate("我晚点给你发消息", -0.10),
        candidate("我晚一点给你发消息", -0.11),
        candidate("等我回来再联系你", -0.16),
        candidate("处理完以后回复你", -0.18),
    ]
    texts = [item.text for item in select_top_candidates(items, count=3, diversity_lambda=0.8)]
    assert texts[0] == "我晚点给你发消息"
    assert "等我回来再联系你" in texts
    assert "处理完以后回复你" in texts


def test_ngram_similarity_is_bounded() -> None:
    assert 0.0 < ngram_similarity("我晚点回复你", "我晚一点回复你") < 1.0


def test_token_longest_common_prefix_handles_retokenized_tail() -> None:
    assert token_longest_common_prefix([1, 2, 3, 4], [1, 2, 8]) == 2
    assert token_longest_common_prefix([1, 2], [1, 2, 3]) == 2


def test_generation_config_rejects_invalid_settings() -> None:
    with pytest.raises(ValueError, match="max_sampling_attempts"):
        ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=7).validate()
    with pytest.raises(ValueError, match="min_new_tokens"):
        ImeGenerationConfig(max_new_tokens=2, min_new_tokens=3).validate()
    with pytest.raises(ValueError, match="temperatures must be positive"):
        ImeGenerationConfig(temperature=0.0).validate()


def test_candidate_pool_stats_count_invalid_and_display_duplicates() -> None:
    items = [candidate("我马上回去", -0.1), candidate("我马上回去。", -0.2), candidate("我晚点回去", -0.3),
             invalid_candidate("我等会再")]
    stats = candidate_pool_stats(items)
    assert (stats.attempts, stats.valid_candidates, stats.valid_unique_candidates) == (4, 3, 2)
    assert (stats.invalid_candidates, stats.duplicate_candidates) == (1, 1)


def test_adaptive_refill_scales_with_filtered_unique_yield() -> None:
    config = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=24, refill_batch_size=8)
    duplicate_heavy = [candidate("我马上回去", -0.1)] * 4 + [invalid_candidate(f"坏候选{i}") for i in range(4)]
    assert adaptive_refill_attempts(duplicate_heavy, config, 8) == 8
    two_unique = [candidate("我马上回去", -0.1), candidate("我晚点回去", -0.2),
                  *[invalid_candidate(f"坏候选{i}") for i in range(6)]]
    assert adaptive_refill_attempts(two_unique, config, 8) == 4
    full = [candidate("我马上回去", -0.1), candidate("我晚点回去", -0.2), candidate("我明天回去", -0.3)]
    assert adaptive_refill_attempts(full, config, 8) == 0


def test_adaptive_refill_respects_remaining_attempt_budget() -> None:
    config = ImeGenerationConfig(max_sampling_attempts=10)
    assert adaptive_refill_attempts([invalid_candidate(f"坏候选{i}") for i in range(8)], config, 8) == 2


def test_refill_schedule_matches_reference_arithmetic() -> None:
    cfg = ImeGenerationConfig()
    assert cfg.refill_schedule(1) == (0.75, 96, 0.95)
    t, k, p = cfg.refill_schedule(2)
    assert abs(t - 0.85) < 1e-12 and k == 128
    t, k, _ = cfg.refill_schedule(5)
    assert t == 0.95 and k == 160


def tiny_config(**changes) -> ModelConfig:
    values = dict(num_layers=8, num_qo_heads=2, num_kv_heads=1, head_dim=64, hidden_size=128, vocab_size=32,
                  intermediate_size=128, hidden_act="silu", rms_norm_eps=1e-6, rope_theta=100_000.0,
                  max_position_embeddings=32, tie_word_embeddings=True, model_type="minimind_ime_v3",
                  architecture_revision="tiny_block_attnres", residual_type="block_attnres", attnres_num_blocks=2,
                  attnres_alpha=1.0)
    values.update(changes)
    return ModelConfig(**values)


def test_attnres_config_rejects_partial_migration_and_bad_partition() -> None:
    with pytest.raises(ValueError, match="alpha=1.0"):
        tiny_config(attnres_alpha=0.5)
    with pytest.raises(ValueError, match="divisible"):
        tiny_config(num_layers=7)
    with pytest.raises(ValueError, match="attnres_backend must be 'reference', 'eager', 'compiled', 'triton'"):
        tiny_config(attnres_backend="flash")


@pytest.mark.parametrize("name", ["reference", "eager", "compiled", "triton", "b200"])
def test_attnres_backend_accepts_reference_names(name) -> None:
    """The reference's AttnRes backend names (aios/models/config.py:27,34-40) are
    all accepted, kept as given, and served by the one sm_100a mixer."""
    from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM

    cfg = tiny_config(attnres_backend=name)
    assert cfg.attnres_backend == name
    with torch.device("meta"):
        model = MiniMindIMEForCausalLM(cfg)
    assert model.model.layers.op_list[0].attn_res_mixer._backend == name
    assert ModelConfig.__dataclass_fields__["attnres_backend"].default == "triton"


def test_cache_manager_fifo_exhaustion_and_double_free() -> None:
    """The free-slot FIFO of aios/scheduler/cache.py:9-51 on a CPU ring: ids come
    out in arange order, frees append at the tail, asking for more than is free
    raises the reference's NotImplementedError (leaving the list untouched), and
    returning more ids than the pool holds is refused."""
    from aios_b200.scheduler.cache import CacheManager

    cm = CacheManager(torch.device("cpu"), 8)
    assert cm.available_size == 8
    a = cm.allocate(3)
    assert a.tolist() == [0, 1, 2] and a.dtype == torch.int32
    b = cm.allocate(4)
    assert b.tolist() == [3, 4, 5, 6] and cm.available_size == 1
    with pytest.raises(NotImplementedError, match="CacheManager eviction is not implemented."):
        cm.allocate(2)
    assert cm.available_size == 1  # a failed allocation takes nothing
    cm._free(a)  # appended after 7, in the order returned
    assert cm.available_size == 4
    assert cm.allocate(4).tolist() == [7, 0, 1, 2]
    cm._free(torch.tensor([5, 3], dtype=torch.int32))
    cm._free([])
    assert cm.allocate(2).tolist() == [5, 3]
    cm._free(list(range(8)))  # everything back: the pool is full
    assert cm.available_size == 8
    with pytest.raises(RuntimeError, match="double free"):
        cm._free([3])
    with pytest.raises(ValueError):
        cm.allocate(-1)
    # the ring mirrors the host list: the next 8 ids in FIFO order
    assert [int(cm.ring[(cm.head + i) % 8]) for i in range(8)] == list(range(8))


def test_attnres_model_state_dict_preserves_checkpoint_names() -> None:
    from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM

    with torch.device("meta"):
        model = MiniMindIMEForCausalLM(tiny_config())
    names = set(model.state_dict())
    assert "model.layers.0.attn_res_mixer.query" in names
    assert "model.layers.7.mlp_res_mixer.key_norm.weight" in names
    assert "model.final_attn_res_mixer.query" in names
    assert "lm_head.weight" not in names
    assert model.model._layers_per_block == 4
    assert model.model._num_blocks == 2


def test_product_kernels_refuse_cpu_tensors() -> None:
    """No CPU fallback: every kernel wrapper rejects host tensors."""
    from aios_b200.kernel import b200_attnres_mix, ops

    with pytest.raises(ValueError, match="CUDA"):
        b200_attnres_mix(torch.zeros(2, 3, 8), None, torch.zeros(8), 1e-6)
    with pytest.raises(ValueError, match="CUDA"):
        ops.linear(torch.zeros(2, 64, dtype=torch.bfloat16), torch.zeros(128, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        ops.rmsnorm(torch.zeros(2, 8), torch.ones(8), 1e-6)


def test_mmr_selection_matches_direct_restatement() -> None:
    """The incremental MMR (cached bigram sets, running maximum similarity) picks
    exactly what the direct form picks: for every round, the first pool entry
    maximising base_score - lambda * max similarity to the chosen ones."""
    import random

    from aios_b200.ime_text import ngram_similarity as sim

    rng = random.Random(7)
    alphabet = "我你他的是了在有一个不这人们来到上大为和国地以中要会"
    for trial in range(200):
        items = []
        for i in range(rng.randint(1, 24)):
            text = "".join(rng.choice(alphabet) for _ in range(rng.randint(2, 7)))
            score = rng.choice([rng.uniform(-3, 0), -1.5, -2.0])  # repeated scores exercise ties
            items.append(ImeCandidate(text=text, token_count=len(text), average_logprob=score, base_score=score,
                                      selection_score=score, stop_reason="eos", invalid_reasons=()))
        lam = rng.choice([0.0, 0.35, 0.8, 2.0])
        count = rng.randint(1, 5)
        got = [(c.text, c.selection_score) for c in select_top_candidates(items, count=count, diversity_lambda=lam)]
        best = {}
        for c in items:
            key = candidate_key(c.text)
            if key not in best or c.base_score > best[key].base_score:
                best[key] = c
        pool, chosen, scores = list(best.values()), [], []
        while pool and len(chosen) < count:
            def mmr(c):
                return c.base_score - lam * max((sim(c.text, x.text) for x in chosen), default=0.0)
            pick = max(pool, key=mmr)
            scores.append(mmr(pick))
            chosen.append(pick)
            pool.remove(pick)
        assert got == [(c.text, s) for c, s in zip(chosen, scores)], trial


def test_repeated_ngram_matches_direct_restatement() -> None:
    """The regex repeat check equals the direct scan of the reference's filter:
    a character four times in a row, or a 2-4 character unit three times."""
    import random

    from aios_b200.ime_text import REPEAT_PATTERN, _repeated_ngram_compact

    def direct(compact: str) -> bool:
        if REPEAT_PATTERN.search(compact):
            return True
        for width in (2, 3, 4):
            for start in range(max(0, len(compact) - 3 * width + 1)):
                unit = compact[start : start + width]
                if unit and compact[start : start + 3 * width] == unit * 3:
                    return True
        return False

    rng = random.Random(0)
    alphabet = "你好天气很不错的了吗。"
    cases = ["", "a", "哈哈哈哈", "你好你好你好", "今天天气很好", "abcabcab", "abcabcabc", "abcdabcdabcd", "ababa"]
    for _ in range(3000):
        n = rng.randint(0, 14)
        text = "".join(rng.choice(alphabet[: rng.randint(2, len(alphabet))]) for _ in range(n))
        if rng.random() < 0.3 and n >= 2:  # plant a repeated unit
            w = rng.randint(2, 4)
            pos = rng.randint(0, n)
            text = text[:pos] + text[:w] * rng.randint(2, 3) + text[pos:]
        cases.append(text)
    for text in cases:
        assert _repeated_ngram_compact(text) == direct(text), text


def test_prefill_tiles_partition_every_request() -> None:
    """The prefill tile list covers each request's new tokens exactly once, in
    order: the fused prefill stores a token's K/V from the one tile that owns it.
    The packed array is [q_start | q_len | cached_len | table_row | tile_req | tile_q0]."""
    from aios_b200.kernel import ops

    for tile in (1, 2, 8):
        for q_lens in ([13], [1, 64, 7], [5, 5, 5, 33], [64] * 3):
            cached = [3 * i for i in range(len(q_lens))]
            rows = list(range(len(q_lens)))[::-1]
            meta, ntiles = ops.prefill_meta(q_lens, cached, rows, tile)
            r = len(q_lens)
            assert len(meta) == 4 * r + 2 * ntiles
            q_start, lens, cl, tr = meta[:r], meta[r : 2 * r], meta[2 * r : 3 * r], meta[3 * r : 4 * r]
            tile_req, tile_q0 = meta[4 * r : 4 * r + ntiles], meta[4 * r + ntiles :]
            assert lens == q_lens and cl == cached and tr == rows
            assert q_start == [sum(q_lens[:i]) for i in range(r)]
            owned = {i: [] for i in range(r)}
            for req, q0 in zip(tile_req, tile_q0):
                owned[req].extend(range(q0, min(q0 + tile, q_lens[req])))
            assert all(owned[i] == list(range(q_lens[i])) for i in range(r))
