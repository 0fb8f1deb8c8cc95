"""Host-side candidate logic of the IME engine (aios/ime.py:17-370).

Text normalisation, hard filters, the soft penalty, display keys, MMR Top-3
selection and the adaptive refill plan. This is CPU string work on at most a few
dozen short candidates per keystroke, so it stays host Python with the
reference's contract; the pattern tables below are the reference's data and
must stay identical for identical filtering.
"""

from __future__ import annotations

import math
import re
from functools import lru_cache
from dataclasses import asdict, dataclass
from typing import Any

ASSISTANT_PATTERN = re.compile(r"以下是|首先|其次|综上所述|作为(?:一个)?AI|我是AI|我来回答")
REPEAT_PATTERN = re.compile(r"(.)\1{3,}")
TERMINAL_TEXT_PATTERN = re.compile(r"[。！？!?；;]")
WHITESPACE_PATTERN = re.compile(r"\s+")
REDUPLICATION_PATTERN = re.compile(r"([\u3400-\u9fff])\1")
# a unit of 2-4 characters repeated three times in a row
TRIPLE_UNIT_PATTERN = re.compile(r"(.{2,4})\1\1", re.DOTALL)
FUNCTION_WORD_ENDINGS = (
    "的", "地", "得", "和", "与", "或", "但", "而", "在", "把", "被", "给",
    "对", "从", "向", "为", "再", "就", "会", "能", "如果", "因为", "所以",
    "但是", "然后",
)
NATURAL_REDUPLICATIONS = frozenset({
    "看看", "想想", "试试", "说说", "问问", "等等", "慢慢", "好好", "聊聊",
    "找找", "改改", "查查", "走走", "听听", "读读", "写写", "帮帮", "常常",
    "刚刚", "轻轻", "渐渐", "偷偷", "偏偏", "仅仅", "人人", "天天",
})
DISPLAY_PUNCTUATION = "，。！？；：,.!?;:"
CJK_LOW, CJK_HIGH = "\u3400", "\u9fff"


@dataclass(frozen=True)
class ImeGenerationConfig:
    display_candidates: int = 3
    sampling_attempts: int = 8
    max_sampling_attempts: int = 24
    refill_batch_size: int = 8
    min_refill_batch_size: int = 2
    max_new_tokens: int = 12
    min_new_tokens: int = 2
    max_candidate_chars: int = 32
    temperature: float = 0.35
    top_k: int = 50
    top_p: float = 0.9
    refill_temperature: float = 0.75
    refill_temperature_step: float = 0.10
    max_refill_temperature: float = 0.95
    refill_top_k: int = 96
    refill_top_k_step: int = 32
    max_refill_top_k: int = 160
    refill_top_p: float = 0.95
    refill_avoid_exact_repeats: bool = True
    refill_ban_min_prefix_tokens: int = 2
    refill_deadline_ms: float = 0.0
    diversity_lambda: float = 0.35
    seed: int = 20260814

    def validate(self) -> None:
        """Same rules and messages as aios/ime.py:58-96."""
        checks = (
            (self.display_candidates >= 1, "display_candidates must be positive"),
            (self.sampling_attempts >= self.display_candidates, "sampling_attempts must cover display_candidates"),
            (self.max_sampling_attempts >= self.sampling_attempts,
             "max_sampling_attempts must cover the initial attempts"),
            (self.refill_batch_size >= 1, "refill_batch_size must be positive"),
            (1 <= self.min_refill_batch_size <= self.refill_batch_size,
             "min_refill_batch_size must be within refill_batch_size"),
            (self.max_new_tokens >= 1, "max_new_tokens must be positive"),
            (0 <= self.min_new_tokens <= self.max_new_tokens, "min_new_tokens must be within max_new_tokens"),
            (0.0 < self.top_p <= 1.0, "top_p must be in (0, 1]"),
            (0.0 < self.refill_top_p <= 1.0, "refill_top_p must be in (0, 1]"),
            (self.temperature > 0.0 and self.refill_temperature > 0.0,
             "IME candidate sampling temperatures must be positive"),
            (self.refill_temperature_step >= 0.0, "refill_temperature_step must be non-negative"),
            (self.max_refill_temperature >= self.refill_temperature,
             "max_refill_temperature must cover refill_temperature"),
            (self.top_k >= 1 and self.refill_top_k >= 1, "IME candidate top_k values must be positive"),
            (self.refill_top_k_step >= 0, "refill_top_k_step must be non-negative"),
            (self.max_refill_top_k >= self.refill_top_k, "max_refill_top_k must cover refill_top_k"),
            (self.refill_deadline_ms >= 0.0, "refill_deadline_ms must be non-negative"),
            (self.refill_ban_min_prefix_tokens >= 1, "refill_ban_min_prefix_tokens must be positive"),
        )
        for ok, message in checks:
            if not ok:
                raise ValueError(message)

    def refill_schedule(self, refill_round: int) -> tuple[float, int, float]:
        """(temperature, top_k, top_p) of refill round 1, 2, ... (aios/ime.py:525-536)."""
        temperature = min(self.max_refill_temperature,
                          self.refill_temperature + (refill_round - 1) * self.refill_temperature_step)
        top_k = min(self.max_refill_top_k, self.refill_top_k + (refill_round - 1) * self.refill_top_k_step)
        return temperature, top_k, self.refill_top_p


@dataclass(frozen=True)
class ImeCandidate:
    text: str
    token_count: int
    average_logprob: float
    base_score: float
    selection_score: float
    stop_reason: str
    invalid_reasons: tuple[str, ...]


@dataclass(frozen=True)
class ImeCompletionResult:
    prefix: str
    generation_id: int
    cancelled: bool
    candidates: tuple[ImeCandidate, ...]
    raw_candidates: tuple[ImeCandidate, ...]
    prefix_tokens: int
    sampling_attempts: int
    generated_tokens: int
    active_model_tokens: int
    latency_ms: float
    gpu_latency_ms: float
    unique_kv_pages: int
    reused_prefix_tokens: int
    refill_rounds: int
    valid_unique_candidates: int
    invalid_candidates: int
    duplicate_candidates: int
    refill_stop_reason: str

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass(frozen=True)
class ImeCandidateScore:
    text: str
    token_count: int
    average_logprob: float
    sum_logprob: float


@dataclass(frozen=True)
class CandidatePoolStats:
    attempts: int
    valid_candidates: int
    valid_unique_candidates: int
    invalid_candidates: int
    duplicate_candidates: int


@dataclass(frozen=True)
class ImeScoringResult:
    prefix: str
    candidates: tuple[ImeCandidateScore, ...]
    latency_ms: float
    gpu_latency_ms: float
    unique_kv_pages: int
    reused_prefix_tokens: int

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def token_longest_common_prefix(left: list[int], right: list[int]) -> int:
    n = 0
    for a, b in zip(left, right):
        if a != b:
            break
        n += 1
    return n


@lru_cache(maxsize=4096)
def normalize_candidate(text: str) -> str:
    # pure; cached because one keystroke normalises each candidate several times
    return WHITESPACE_PATTERN.sub("", text.replace("\ufffd", "")).strip()


def truncate_at_terminal(text: str) -> tuple[str, bool]:
    """Cut after the first sentence terminator (commas do not end an IME phrase)."""
    found = TERMINAL_TEXT_PATTERN.search(text)
    if found is None:
        return text, False
    return text[: found.end()], True


@lru_cache(maxsize=4096)
def candidate_key(text: str) -> str:
    return normalize_candidate(text).rstrip(DISPLAY_PUNCTUATION).casefold()


def repeated_ngram(text: str) -> bool:
    return _repeated_ngram_compact(normalize_candidate(text))


def _repeated_ngram_compact(compact: str) -> bool:
    # a character four times in a row, or a 2-4 character unit three times
    return REPEAT_PATTERN.search(compact) is not None or TRIPLE_UNIT_PATTERN.search(compact) is not None


def invalid_reasons(text: str, config: ImeGenerationConfig, prefix: str = "") -> tuple[str, ...]:
    compact = normalize_candidate(text)
    if not compact:
        return ("empty",)
    reasons: list[str] = []
    if len(compact) < 2:
        reasons.append("too_short")
    if config.max_candidate_chars > 0 and len(compact) > config.max_candidate_chars:
        reasons.append("too_long")
    if ASSISTANT_PATTERN.search(compact):
        reasons.append("assistant_template")
    if _repeated_ngram_compact(compact):
        reasons.append("repeated_ngram")
    if compact.rstrip(DISPLAY_PUNCTUATION).endswith(FUNCTION_WORD_ENDINGS):
        reasons.append("unfinished_fragment")
    # A doubled CJK character across the join (你好 + 好好休息) is rejected; a
    # single repeat (今天 + 天气很好) is natural and allowed.
    if prefix and CJK_LOW <= prefix[-1] <= CJK_HIGH and compact.startswith(prefix[-1] * 2):
        reasons.append("boundary_repeat")
    return tuple(reasons)


def soft_penalty(text: str) -> float:
    compact = normalize_candidate(text)
    penalty = 0.0
    for match in REDUPLICATION_PATTERN.finditer(compact):
        if match.group(0) not in NATURAL_REDUPLICATIONS:
            penalty += 0.45
    if len(compact) <= 3:
        penalty += 0.08
    return penalty


def _grams(text: str, width: int = 2) -> set[str]:
    compact = candidate_key(text)
    if len(compact) < width:
        return {compact} if compact else set()
    return {compact[i : i + width] for i in range(len(compact) - width + 1)}


def _jaccard(a: set[str], b: set[str]) -> float:
    if not a or not b:
        return 0.0
    return len(a & b) / len(a | b)


def ngram_similarity(left: str, right: str, width: int = 2) -> float:
    return _jaccard(_grams(left, width), _grams(right, width))


def _valid(candidate: ImeCandidate) -> bool:
    return not candidate.invalid_reasons and math.isfinite(candidate.base_score)


def select_top_candidates(candidates: list[ImeCandidate], count: int, diversity_lambda: float) -> list[ImeCandidate]:
    """Best candidate per display key, then greedy MMR: score - lambda * max
    bigram-Jaccard similarity to the already selected ones."""
    best: dict[str, ImeCandidate] = {}
    for cand in candidates:
        if not _valid(cand):
            continue
        key = candidate_key(cand.text)
        held = best.get(key)
        if held is None or cand.base_score > held.base_score:
            best[key] = cand
    pool = list(best.values())
    # bigram sets computed once per candidate; each pool entry keeps its running
    # maximum similarity to the chosen ones, updated against the newest pick only
    grams = [_grams(c.text) for c in pool]
    max_sim = [0.0] * len(pool)
    alive = list(range(len(pool)))
    chosen: list[ImeCandidate] = []
    while alive and len(chosen) < count:
        # the first entry with the largest MMR score (as max() picks it)
        pick_i = alive[0]
        score = pool[pick_i].base_score - diversity_lambda * max_sim[pick_i]
        for i in alive[1:]:
            value = pool[i].base_score - diversity_lambda * max_sim[i]
            if value > score:
                pick_i, score = i, value
        alive.remove(pick_i)
        picked = grams[pick_i]
        if picked:
            for i in alive:
                other = grams[i]
                if other:
                    sim = len(other & picked) / len(other | picked)
                    if sim > max_sim[i]:
                        max_sim[i] = sim
        pick = pool[pick_i]
        chosen.append(ImeCandidate(
            text=pick.text, token_count=pick.token_count, average_logprob=pick.average_logprob,
            base_score=pick.base_score, selection_score=score, stop_reason=pick.stop_reason,
            invalid_reasons=pick.invalid_reasons,
        ))
    return chosen


def candidate_pool_stats(candidates: list[ImeCandidate]) -> CandidatePoolStats:
    valid = [c for c in candidates if _valid(c)]
    unique = {candidate_key(c.text) for c in valid}
    return CandidatePoolStats(
        attempts=len(candidates),
        valid_candidates=len(valid),
        valid_unique_candidates=len(unique),
        invalid_candidates=len(candidates) - len(valid),
        duplicate_candidates=len(valid) - len(unique),
    )


def adaptive_refill_attempts(candidates: list[ImeCandidate], config: ImeGenerationConfig, attempts_used: int) -> int:
    """Fresh branches for the filtered Top-3 deficit: enough to cover it at the
    observed unique-valid yield (floored at 1/refill_batch_size), at least twice
    the deficit and the configured minimum, capped by the batch and the budget."""
    remaining = config.max_sampling_attempts - attempts_used
    if remaining <= 0:
        return 0
    stats = candidate_pool_stats(candidates)
    deficit = config.display_candidates - stats.valid_unique_candidates
    if deficit <= 0:
        return 0
    floor = 1.0 / max(1, config.refill_batch_size)
    observed = stats.valid_unique_candidates / stats.attempts if stats.attempts else floor
    predicted = math.ceil(deficit / max(floor, observed))
    planned = max(config.min_refill_batch_size, 2 * deficit, predicted)
    return min(planned, config.refill_batch_size, remaining)
