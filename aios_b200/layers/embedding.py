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

    @staticmethod
    def _select(batch, *tensors):
        """Rows the logits are needed for (the last token of each prefill request)."""
        if not (batch.is_prefill and not batch.return_all_logits):
            return tensors
        md = batch.attn_metadata
        rows = getattr(md, "last_rows", ())
        if len(rows) == 1:  # one request: views, no gather
            return tuple(None if t is None else t[rows[0] : rows[0] + 1] for t in tensors)
        idx = md.get_last_indices(batch.size)
        return tuple(None if t is None else t.index_select(0, idx) for t in tensors)

    def _w(self) -> torch.Tensor:
        return self._tied_embedding.weight if self._tie_word_embeddings else self.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        (x,) = self._select(batch, x)
        return ops.linear(x.contiguous(), self._w(), out=batch.logits_out)

    def forward_normed(self, x: torch.Tensor, residual: torch.Tensor | None, norm_weight: torch.Tensor,
                       eps: float) -> torch.Tensor:
        """LM head on rmsnorm(x + residual) * norm_weight, computed only for the
        rows that need logits (the last token of each prefill request)."""
        batch = get_global_ctx().batch
        x, residual = self._select(batch, x, residual)
        if residual is None:
            h = ops.rmsnorm(x.contiguous(), norm_weight, eps)
        else:
            h = x.contiguous().clone() if not x.is_contiguous() else x
            r = residual.contiguous().clone() if not residual.is_contiguous() else residual
            ops.fused_add_rmsnorm(h, r, norm_weight, eps)
        w = self._w()
        tiles = batch.tile_stats_out
        if tiles is not None and batch.is_decode and ops.tile_stats_eligible(h.shape[0], w.shape[1], w.shape[0]):
            batch.tile_stats_written = True
            return ops.linear(h, w, out=batch.logits_out, tile_stats=tiles)
        return ops.linear(h, w, out=batch.logits_out)

    def forward_stat(self, stats: ops.RowStats, norm_weight: torch.Tensor, eps: float) -> torch.Tensor:
        """LM head on the final RMSNorm of a residual stream given by its
        statistics, for the rows that need logits only."""
        batch = get_global_ctx().batch
        if batch.is_prefill and not batch.return_all_logits:
            md = batch.attn_metadata
            rows = getattr(md, "last_rows", ())
            if len(rows) == 1:
                stats = stats.rows(rows[0], rows[0] + 1)
            else:
                stats = stats.select(md.get_last_indices(batch.size))
        tiles = batch.tile_stats_out
        w = self._w()
        if tiles is not None and batch.is_decode and ops.tile_stats_eligible(stats.x.shape[0], w.shape[1], w.shape[0]):
            batch.tile_stats_written = True
            return ops.linear_stat_norm(stats, norm_weight, eps, w, out=batch.logits_out, tile_stats=tiles)
        return ops.linear_stat_norm(stats, norm_weight, eps, w, out=batch.logits_out)

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
