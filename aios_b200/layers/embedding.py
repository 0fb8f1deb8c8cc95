"""Embedding and LM head (aios/layers/embedding.py:13-65) on the sm_100a kernels."""

from __future__ import annotations

from typing import Dict

import torch

from ..core import get_global_ctx
from ..kernel import ops
from .base import BaseOP, _concat_prefix


class Embedding(BaseOP):
    def __init__(self, num_embeddings: int, embedding_dim: int):
        self.weight = torch.empty(num_embeddings, embedding_dim)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return ops.embedding(input_ids, self.weight)


class LMHead(BaseOP):
    def __init__(
        self,
        num_embeddings: int,
        embedding_dim: int,
        tie_word_embeddings: bool = False,
        tied_embedding: Embedding | None = None,
    ):
        self._tie_word_embeddings = tie_word_embeddings
        self._tied_embedding = tied_embedding
        if not tie_word_embeddings:
            self.weight = torch.empty(num_embeddings, embedding_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        if batch.is_prefill and not batch.return_all_logits:
            md = batch.attn_metadata
            rows = getattr(md, "last_rows", ())
            if len(rows) == 1:
                x = x[rows[0] : rows[0] + 1]  # one request: a view, no gather
            else:
                x = x.index_select(0, md.get_last_indices(batch.size))
        w = self._tied_embedding.weight if self._tie_word_embeddings else self.weight
        return ops.linear(x.contiguous(), w, out=batch.logits_out)

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *, prefix: str = "", _internal: bool = False) -> None:
        if self._tie_word_embeddings:
            key = _concat_prefix(prefix, "weight")
            if key in state_dict:
                state_dict.pop(key)
        else:
            super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)

    def state_dict(self, *, prefix: str = "") -> Dict[str, torch.Tensor]:
        if self._tie_word_embeddings:
            return {}
        return super().state_dict(prefix=prefix)
