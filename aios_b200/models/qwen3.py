"""Standard-residual decoder (aios/models/qwen3.py:31-173) on the sm_100a kernels.

Per layer and forward (``forward_stat``, the path the B200 backend runs): qkv
GEMM that normalises its own input from the residual statistics, the attention
kernel that also applies q/k RMSNorm + bf16 RoPE and writes the new K/V, o GEMM
whose epilogue adds the residual and emits the next statistics, gate/up GEMM
(normalising input, SwiGLU epilogue), down GEMM (residual add + statistics).
RMSNormFused (aios/layers/norm.py:34-40) is thereby split across the GEMM before
and the GEMM after it, and no normalised tensor is written. ``forward`` keeps the
reference's call structure for any other attention backend. The parameter
names and their order equal the reference's, so checkpoints load unchanged.
"""

from __future__ import annotations

import os
from typing import TYPE_CHECKING

import torch

from ..attention import B200AttentionBackend, BaseAttentionBackend
from .. import _lib
from ..core import get_global_ctx
from ..kernel import ops
from ..layers import (
    BaseOP,
    Embedding,
    Linear,
    LinearColParallelMerged,
    LinearQKVMerged,
    LMHead,
    OPList,
    RMSNorm,
    RMSNormFused,
    RotaryEmbedding,
)
from .base import BaseLLMModel

if TYPE_CHECKING:
    from ..core import Batch
    from ..kvcache import MHAKVCache
    from .config import ModelConfig


# The gate/up linears, and the qkv linears from the second layer on, let their
# successor launch before their own dependency wait, so that the decode
# attention's key-history staging (and the down linear's weight loads) overlap
# them. Per layer in place on the S10 decode step (qkv, attention, o, gate/up,
# down; us): 2.91 3.33 1.70 3.36 2.14 = 13.44 before, 2.11 3.26 1.76 3.10 2.53 =
# 12.76 after (qkv alone early: 12.92). AIOSB_EARLY_LINEARS=0 keeps the launch
# after the wait.
_EARLY_LINEARS = os.environ.get("AIOSB_EARLY_LINEARS", "1") != "0"


class Qwen3Attention(BaseOP):
    def __init__(self, config: ModelConfig, layer_idx: int, attn_backend: BaseAttentionBackend):
        self.num_heads = config.num_qo_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self._layer_idx = layer_idx
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.qkv_proj = LinearQKVMerged(config.hidden_size, self.q_size, self.kv_size)
        self.o_proj = Linear(self.num_heads * self.head_dim, config.hidden_size)
        self.q_norm = RMSNorm(self.head_dim, config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, config.rms_norm_eps)
        self._attn_backend = attn_backend

    def attend(self, hidden_states: torch.Tensor, rotary: RotaryEmbedding, paged_kv_cache: MHAKVCache,
               batch: Batch) -> torch.Tensor:
        """Projection + attention, without o_proj: [T, Hq * d]."""
        return self.attend_qkv(self.qkv_proj.forward(hidden_states), rotary, paged_kv_cache, batch)

    def attend_qkv(self, qkv: torch.Tensor, rotary: RotaryEmbedding, paged_kv_cache: MHAKVCache,
                   batch: Batch) -> torch.Tensor:
        """Attention on a packed [T, (Hq + 2 Hkv) * d] projection: [T, Hq * d]."""
        backend = self._attn_backend
        if isinstance(backend, B200AttentionBackend):
            cos, sin = rotary.tables()
            return backend.forward_qkv(
                qkv, self.q_norm.weight, self.k_norm.weight, cos, sin, paged_kv_cache, self._layer_idx, batch
            )
        # A third-party backend plugged into the reference slot gets normalised,
        # rotated q/k and v as aios/models/qwen3.py:61-73 hands them over, and stores
        # K/V itself (aios/attention/base.py:23-28). The q/k norm and RoPE run on the
        # prefill prologue kernel, with k and v written to a per-call token buffer
        # (slot t = token t) instead of the cache.
        tokens = qkv.shape[0]
        dev = qkv.device
        cos, sin = rotary.tables()
        q = torch.empty(tokens, self.num_heads, self.head_dim, dtype=qkv.dtype, device=dev)
        k = torch.empty(tokens, self.num_kv_heads, self.head_dim, dtype=qkv.dtype, device=dev)
        v = torch.empty_like(k)
        ops.qk_norm_rope_store(
            qkv=qkv, num_qo_heads=self.num_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
            q_norm_w=self.q_norm.weight, k_norm_w=self.k_norm.weight, eps=self.q_norm.eps, cos=cos, sin=sin,
            positions=batch.positions.to(torch.int32).contiguous(),
            out_loc=torch.arange(tokens, dtype=torch.int32, device=dev), k_cache=k, v_cache=v,
            q_out=q.view(tokens, -1),
        )
        return backend.forward(q, k, v, paged_kv_cache, self._layer_idx, batch).reshape(tokens, -1)

    def forward(self, hidden_states, rotary, paged_kv_cache, batch) -> torch.Tensor:
        return self.o_proj.forward(self.attend(hidden_states, rotary, paged_kv_cache, batch))


class Qwen3MLP(BaseOP):
    def __init__(self, config: ModelConfig):
        self.gate_up_proj = LinearColParallelMerged(
            config.hidden_size, [config.intermediate_size, config.intermediate_size]
        )
        self.down_proj = Linear(config.intermediate_size, config.hidden_size)
        if config.hidden_act != "silu":
            raise ValueError(f"Unsupported activation: {config.hidden_act}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj.forward(self.gate_up_proj.forward_silu_mul(x))


class Qwen3DecoderLayer(BaseOP):
    def __init__(self, config: ModelConfig, layer_idx: int, attn_backend: BaseAttentionBackend):
        self.self_attn = Qwen3Attention(config, layer_idx, attn_backend)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    def forward(self, hidden_states, rotary, paged_kv_cache, batch, residual):
        hidden_states, residual = self.input_layernorm.forward(hidden_states, residual)
        hidden_states = self.self_attn.forward(hidden_states, rotary, paged_kv_cache, batch)
        hidden_states, residual = self.post_attention_layernorm.forward(hidden_states, residual)
        return self.mlp.forward(hidden_states), residual

    def forward_stat(self, stats: ops.RowStats, residual: torch.Tensor, rotary, paged_kv_cache,
                     batch) -> ops.RowStats:
        """The same layer with both norms folded into the GEMMs: ``stats`` describe
        the residual stream entering the layer, ``residual`` (bf16, updated in
        place) is that stream rounded; returns the statistics leaving it."""
        attn, mlp = self.self_attn, self.mlp
        n1, n2 = self.input_layernorm, self.post_attention_layernorm
        # Early launch of the successor (see _EARLY_LINEARS). The gate/up
        # linear's successor, the down linear, reads only its weights before its
        # wait. The qkv linear's successor, the decode attention, reads row
        # metadata and key history before its wait; from the second layer on it
        # can start only after the previous layer's attention passed its wait
        # (that kernel launches its successor only then), so every kernel up to
        # the previous layer's qkv, the group step included, has completed. The
        # first layer's qkv follows the embedding, whose predecessor is the group
        # step itself.
        qkv = ops.linear_stat_norm(stats, n1.weight, n1.eps, attn.qkv_proj.weight,
                                   early_dependents=_EARLY_LINEARS and attn._layer_idx > 0)
        a = attn.attend_qkv(qkv, rotary, paged_kv_cache, batch)
        stats = ops.linear_add_stat(a, attn.o_proj.weight, residual)
        act = ops.linear_stat_norm(stats, n2.weight, n2.eps, mlp.gate_up_proj.packed_weight(),
                                   epilogue=_lib.EPI_SILU_MUL, early_dependents=_EARLY_LINEARS)
        return ops.linear_add_stat(act, mlp.down_proj.weight, residual)


class Qwen3Model(BaseOP):
    def __init__(self, config: ModelConfig):
        self.attn_backend = B200AttentionBackend(config)
        self.embed_tokens = Embedding(config.vocab_size, config.hidden_size)
        self.layers = OPList([Qwen3DecoderLayer(config, i, self.attn_backend) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self._rotary_emb = RotaryEmbedding(config.head_dim, config.max_position_embeddings, config.rope_theta)

    def forward_hidden(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Decoder trunk without the final norm: (hidden, residual)."""
        ctx = get_global_ctx()
        batch = ctx.batch
        hidden_states = self.embed_tokens.forward(batch.input_ids)
        residual: torch.Tensor | None = None
        for layer in self.layers.op_list:
            hidden_states, residual = layer.forward(hidden_states, self._rotary_emb, ctx.kv_cache, batch, residual)
        return hidden_states, residual

    def forward_stats(self) -> ops.RowStats:
        """Decoder trunk with every RMSNorm folded into the GEMMs; returns the
        statistics of the final residual stream (the final norm's input)."""
        ctx = get_global_ctx()
        batch = ctx.batch
        if batch.is_decode and batch.pre_embedded is not None:
            residual, stats = batch.pre_embedded
        else:
            residual, stats = ops.embedding_stat(batch.input_ids, self.embed_tokens.weight)
        for layer in self.layers.op_list:
            stats = layer.forward_stat(stats, residual, self._rotary_emb, ctx.kv_cache, batch)
        return stats

    def forward(self) -> torch.Tensor:
        hidden_states, residual = self.forward_hidden()
        return self.norm.forward(hidden_states, residual)[0]


class Qwen3ForCausalLM(BaseLLMModel):
    def __init__(self, config: ModelConfig):
        self.model = Qwen3Model(config)
        self.attn_backend = self.model.attn_backend
        self.lm_head = LMHead(
            config.vocab_size,
            config.hidden_size,
            tie_word_embeddings=config.tie_word_embeddings,
            tied_embedding=self.model.embed_tokens if config.tie_word_embeddings else None,
        )

    def forward(self) -> torch.Tensor:
        norm = self.model.norm
        if isinstance(self.attn_backend, B200AttentionBackend):
            return self.lm_head.forward_stat(self.model.forward_stats(), norm.weight, norm.eps)
        hidden_states, residual = self.model.forward_hidden()
        return self.lm_head.forward_normed(hidden_states, residual, norm.weight, norm.eps)
