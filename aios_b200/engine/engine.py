"""One batched forward plus per-request sampling for the generic ``LLM.generate``
path (aios/engine/engine.py:15-38)."""

from __future__ import annotations

from typing import TYPE_CHECKING

import torch

from ..core import get_global_ctx
from .sample import Sampler

if TYPE_CHECKING:
    from ..core import Batch
    from ..kvcache import MHAKVCache


class Engine:
    def __init__(self, model, mha_kv_cache: "MHAKVCache") -> None:
        self.model = model
        self.mha_kv_cache = mha_kv_cache

    def run_batch(self, batch: "Batch") -> torch.Tensor:
        """Forward over the batch, then each request's next token with its own
        sampling parameters; requests that share parameters are sampled in one
        sampler launch. Returns the [batch] next-token ids."""
        ctx = get_global_ctx()
        with ctx.forward_batch(batch):
            logits = self.model.forward()
        last = logits[: batch.size]
        next_tokens = torch.empty(batch.size, dtype=torch.int64, device=last.device)
        groups: dict = {}
        for i, req in enumerate(batch.reqs):
            groups.setdefault(repr(req.sampling_params), (req.sampling_params, []))[1].append(i)
        for params, rows in groups.values():
            index = torch.tensor(rows, dtype=torch.int64).to(last.device, non_blocking=True)
            tokens = Sampler(params).sample(last.index_select(0, index))
            next_tokens.index_copy_(0, index, tokens.view(-1))
        return next_tokens
