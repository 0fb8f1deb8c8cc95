"""Runtime data model: the reference's boundary types (aios/core.py:14-125).

``SamplingParams``, ``Req``, ``Batch`` and the process-global ``Context`` keep the
reference's fields and semantics, so model code written against aios reads the
active batch the same way. ``reset_global_ctx`` is an addition for test suites
that build several engines in one process.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, List, Literal

import torch

if TYPE_CHECKING:
    from .attention import BaseAttentionBackend, BaseAttentionMetadata
    from .kvcache import MHAKVCache


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    max_tokens: int = 1024

    @property
    def is_greedy(self) -> bool:
        return (self.temperature <= 0.0 or self.top_k == 1) and self.top_p == 1.0


@dataclass(eq=False)
class Req:
    """Per-request runtime state: tokens [0, cached_len) are in the KV cache,
    [cached_len, device_len) are computed by the next forward."""

    input_ids: torch.Tensor
    cached_len: int
    output_len: int
    uid: int
    sampling_params: SamplingParams
    table_idx: int | None = None
    generated: List[int] = field(default_factory=list)

    def __post_init__(self) -> None:
        self.device_len = len(self.input_ids)
        self.max_device_len = len(self.input_ids) + self.output_len
        assert 0 <= self.cached_len <= self.device_len <= self.max_device_len

    @property
    def remain_len(self) -> int:
        return self.max_device_len - self.device_len

    @property
    def extend_len(self) -> int:
        return self.device_len - self.cached_len

    def complete_one(self) -> None:
        self.cached_len = self.device_len
        self.device_len += 1

    @property
    def can_decode(self) -> bool:
        return self.remain_len > 0


@dataclass
class Batch:
    """Requests of one forward pass; the engine fills input_ids / positions /
    out_loc, the attention backend fills attn_metadata."""

    reqs: List[Req]
    phase: Literal["prefill", "decode"]
    input_ids: torch.Tensor = field(init=False)
    positions: torch.Tensor = field(init=False)
    out_loc: torch.Tensor = field(init=False)
    attn_metadata: "BaseAttentionMetadata" = field(init=False)
    return_all_logits: bool = False
    # Optional preallocated [rows, vocab] buffer the LM head writes into (lets a
    # captured decode step leave its logits where the next sampling step reads).
    logits_out: torch.Tensor | None = None
    # Optional [vocab / 16, rows, 4] fp32 buffer for the LM head's per-16-id tile
    # statistics of the logits (a decode step whose sampler reads them); the LM
    # head sets tile_stats_written when it filled it.
    tile_stats_out: torch.Tensor | None = None
    tile_stats_written: bool = False
    # Optional decode input already embedded (the CandidateGroup step writes it):
    # (bf16 rows [rows, hidden], RowStats of them); the trunk then starts at its
    # first linear instead of the embedding
    pre_embedded: tuple | None = None

    @property
    def is_prefill(self) -> bool:
        return self.phase == "prefill"

    @property
    def is_decode(self) -> bool:
        return self.phase == "decode"

    @property
    def size(self) -> int:
        return len(self.reqs)


@dataclass
class Context:
    page_size: int
    page_table: torch.Tensor = field(init=False)
    attn_backend: "BaseAttentionBackend" = field(init=False)
    kv_cache: "MHAKVCache" = field(init=False)
    _batch: Batch | None = field(default=None, init=False)

    @property
    def batch(self) -> Batch:
        assert self._batch is not None, "No active batch in context"
        return self._batch

    @contextmanager
    def forward_batch(self, batch: Batch):
        assert self._batch is None, "Nested forward_batch is not allowed"
        try:
            self._batch = batch
            yield
        finally:
            self._batch = None


_GLOBAL_CTX: Context | None = None


def set_global_ctx(ctx: Context) -> None:
    global _GLOBAL_CTX
    assert _GLOBAL_CTX is None, "Global context is already set"
    _GLOBAL_CTX = ctx


def get_global_ctx() -> Context:
    assert _GLOBAL_CTX is not None, "Global context is not set"
    return _GLOBAL_CTX


def reset_global_ctx() -> None:
    """Drops the process-global context (one engine per process otherwise)."""
    global _GLOBAL_CTX
    _GLOBAL_CTX = None
