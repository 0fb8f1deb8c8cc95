"""B200-native (sm_100a) AIOS-IME CandidateGroup engine.

Drop-in for the reference package's per-keystroke path: the same public names
(``LLM``, ``ImeCompletionEngine``, ``ImeGenerationConfig``, ``Sampler``, ...) with
every GPU op implemented as a hand-written Blackwell kernel behind the C ABI in
``include/aios_b200.h``.
"""

from .core import SamplingParams
from .engine import Sampler
from .ime import (
    CancellationToken,
    CandidatePoolStats,
    ImeCandidate,
    ImeCandidateScore,
    ImeCompletionEngine,
    ImeCompletionResult,
    ImeGenerationConfig,
    ImeScoringResult,
    adaptive_refill_attempts,
    candidate_pool_stats,
    token_longest_common_prefix,
    truncate_at_terminal,
)
from .llm import LLM

__all__ = [
    "CancellationToken",
    "CandidatePoolStats",
    "ImeCandidate",
    "ImeCandidateScore",
    "ImeCompletionEngine",
    "ImeCompletionResult",
    "ImeGenerationConfig",
    "ImeScoringResult",
    "LLM",
    "Sampler",
    "SamplingParams",
    "adaptive_refill_attempts",
    "candidate_pool_stats",
    "token_longest_common_prefix",
    "truncate_at_terminal",
]
