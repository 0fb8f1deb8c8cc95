"""MiniMind-IME model (aios/models/minimind_ime.py) on the sm_100a kernels.

Standard-residual bundles reuse the Qwen3 decoder. Block AttnRes bundles
(0.214B: 32 layers, 8 blocks, 65 depth mixers) run each mixer as one fused
kernel (RMS score + depth softmax + weighted sum), and fold the block-local
residual adds ``partial + delta`` into the o_proj / down_proj GEMM epilogues;
the last layer of a block writes its partial straight into the bank slot.
"""

from __future__ import annotations

import os

from typing import TYPE_CHECKING

import torch

from .. import _lib
from ..attention import B200AttentionBackend
from ..core import get_global_ctx
from ..kernel import ops
from ..layers import BaseOP, Embedding, LMHead, OPList, RMSNorm, RotaryEmbedding
from .qwen3 import _EARLY_LINEARS, Qwen3Attention, Qwen3ForCausalLM, Qwen3MLP

if TYPE_CHECKING:
    from ..core import Batch
    from ..kvcache import MHAKVCache
    from .config import ModelConfig


class BlockAttnResMixer(BaseOP):
    """Kimi Block AttnRes depth mixer for ``alpha = 1``; weights ``query`` and
    ``key_norm.weight`` as in the reference checkpoints."""

    def __init__(self, hidden_size: int, eps: float, backend: str = "b200") -> None:
        self.query = torch.empty(hidden_size)
        self.key_norm = RMSNorm(hidden_size, eps)
        self._backend = backend
        self._weighted_query: torch.Tensor | None = None

    def on_weights_loaded(self) -> None:
        self._weighted_query = None

    def _routing_query(self) -> torch.Tensor:
        """query * key_norm.weight folded once in fp32 (aios/models/minimind_ime.py:106-117)."""
        cached = self._weighted_query
        if cached is None or cached.device != self.query.device or cached.shape != self.query.shape:
            cached = (self.query.float() * self.key_norm.weight.float()).contiguous()
            self._weighted_query = cached
        return cached

    def forward(
        self,
        bank: torch.Tensor,
        partial: torch.Tensor | None = None,
        *,
        score_buffer: torch.Tensor | None = None,
        output_buffer: torch.Tensor | None = None,
    ) -> torch.Tensor:
        if bank.ndim != 3:
            raise ValueError(f"AttnRes bank must have shape [S,N,D], got {tuple(bank.shape)}")
        if bank.shape[-1] != self.query.numel():
            raise ValueError("AttnRes bank hidden size does not match query")
        if partial is not None and partial.shape != bank.shape[1:]:
            raise ValueError("AttnRes partial must have shape [N,D] matching bank")
        return ops.b200_attnres_mix(
            bank, partial, self._routing_query(), self.key_norm.eps,
            score_buffer=score_buffer, output_buffer=output_buffer,
        )


# AIOSB_FUSED_MIXER=1: in decode (<= 8 tokens) each layer's two mixers and the
# RMSNorms after them run inside the qkv and gate/up linears
# (aiosb_linear_attnres_rmsnorm). Off by default: every CTA of those linears then
# stages the bank rows of all 8 tokens (up to 100 KB) and rebuilds the mixer's
# rows, which measured slower than the mixer kernel it removes (S21 decode
# forward 932 us against 603 us; refill keystroke 45.2 against 30.8 ms; still
# 635 against 612 us when only mixers of at most 2 sources are fused).
_FUSED_MIXER = os.environ.get("AIOSB_FUSED_MIXER", "0") == "1"


def mix_and_norm(mixer: BlockAttnResMixer, norm: RMSNorm, bank: torch.Tensor, partial: torch.Tensor | None,
                 output_buffer: torch.Tensor, stable: int = 0) -> torch.Tensor:
    """norm(mixer(bank, partial)): one kernel when the sources fit the fused form
    (<= 10 sources, hidden <= 768), else the mixer and the norm kernels.

    ``stable``: the first bank sources that were written before the previous
    kernel on the stream began; the fused kernel reads them before waiting on it.
    In the trunk every launch follows its predecessor's launch, and the qkv, the
    attention and the gate/up kernels let their successors launch only after
    their own wait; a mixer therefore starts after every kernel up to the last of
    those has finished. That covers every bank source except one written by the
    kernel just before the mixer: the embedding (block 0), or the down projection
    that closed the previous block (the first mixer of a block, the final one)."""
    sources = bank.shape[0] + (partial is not None)
    if sources <= 10 and bank.shape[-1] <= 768 and bank.shape[-1] % 8 == 0:
        return ops.b200_attnres_mix_rmsnorm(bank, partial, mixer._routing_query(), mixer.key_norm.eps, norm.weight,
                                           norm.eps, output_buffer=output_buffer, stable_sources=stable)
    return norm.forward(mixer.forward(bank, partial, output_buffer=output_buffer))


class MiniMindAttnResDecoderLayer(BaseOP):
    """One attention/MLP pair that contributes deltas to its block's partial."""

    def __init__(self, config: ModelConfig, layer_idx: int, attn_backend: B200AttentionBackend) -> None:
        self.self_attn = Qwen3Attention(config, layer_idx, attn_backend)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.attn_res_mixer = BlockAttnResMixer(config.hidden_size, config.rms_norm_eps, config.attnres_backend)
        self.mlp_res_mixer = BlockAttnResMixer(config.hidden_size, config.rms_norm_eps, config.attnres_backend)

    def forward(
        self,
        bank: torch.Tensor,
        partial: torch.Tensor | None,
        rotary: RotaryEmbedding,
        paged_kv_cache: MHAKVCache,
        batch: Batch,
        mixed: torch.Tensor,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        # without a partial this is a block's first layer, whose newest bank
        # source was written by the kernel just before
        stable = bank.shape[0] if partial is not None else bank.shape[0] - 1
        mixer, norm = self.attn_res_mixer, self.input_layernorm
        if _FUSED_MIXER and ops.linear_attnres_rmsnorm_eligible(bank, partial, stable):
            # decode: the mixer and its norm inside the qkv projection
            qkv = ops.linear_attnres_rmsnorm(bank, partial, stable, mixer._routing_query(), mixer.key_norm.eps,
                                             norm.weight, norm.eps, self.self_attn.qkv_proj.weight)
            attn = self.self_attn.attend_qkv(qkv, rotary, paged_kv_cache, batch)
        else:
            # the mixer writes the input-normalised rows straight away
            normed = mix_and_norm(mixer, norm, bank, partial, mixed, stable)
            # the qkv linear launches the attention early from the second layer
            # on, and the gate/up linear the down linear (qwen3._EARLY_LINEARS)
            qkv = ops.linear(normed, self.self_attn.qkv_proj.weight,
                             early_dependents=_EARLY_LINEARS and self.self_attn._layer_idx > 0)
            attn = self.self_attn.attend_qkv(qkv, rotary, paged_kv_cache, batch)
        w_o = self.self_attn.o_proj.weight
        if partial is None:
            partial = ops.linear(attn, w_o)
        else:
            ops.linear(attn, w_o, out=partial, epilogue=_lib.EPI_ADD, residual=partial)
        mixer, norm = self.mlp_res_mixer, self.post_attention_layernorm
        if _FUSED_MIXER and ops.linear_attnres_rmsnorm_eligible(bank, partial, bank.shape[0]):
            act = ops.linear_attnres_rmsnorm(bank, partial, bank.shape[0], mixer._routing_query(),
                                             mixer.key_norm.eps, norm.weight, norm.eps,
                                             self.mlp.gate_up_proj.packed_weight(), epilogue=_lib.EPI_SILU_MUL)
        else:
            normed = mix_and_norm(mixer, norm, bank, partial, mixed, bank.shape[0])
            act = ops.linear(normed, self.mlp.gate_up_proj.packed_weight(), epilogue=_lib.EPI_SILU_MUL,
                             early_dependents=_EARLY_LINEARS)
        target = partial if out is None else out
        ops.linear(act, self.mlp.down_proj.weight, out=target, epilogue=_lib.EPI_ADD, residual=partial)
        return target


class MiniMindBlockAttnResModel(BaseOP):
    """Inference trunk with block-local deltas and depth routing."""

    def __init__(self, config: ModelConfig) -> None:
        self.attn_backend = B200AttentionBackend(config)
        self.embed_tokens = Embedding(config.vocab_size, config.hidden_size)
        self.layers = OPList(
            [MiniMindAttnResDecoderLayer(config, i, self.attn_backend) for i in range(config.num_layers)]
        )
        self.final_attn_res_mixer = BlockAttnResMixer(config.hidden_size, config.rms_norm_eps, config.attnres_backend)
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self._rotary_emb = RotaryEmbedding(config.head_dim, config.max_position_embeddings, config.rope_theta)
        self._num_blocks = config.attnres_num_blocks
        self._layers_per_block = config.layers_per_attnres_block

    def forward_hidden(self) -> torch.Tensor:
        """Trunk up to the final mixer (before the final norm)."""
        bank, mixed = self._trunk()
        return self.final_attn_res_mixer.forward(bank, output_buffer=mixed)

    def _trunk(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Every block; returns the bank of block outputs and the mixer buffer."""
        ctx = get_global_ctx()
        batch = ctx.batch
        ids = batch.input_ids
        tokens = ids.numel()
        hidden = self.embed_tokens.weight.shape[1]
        bank_storage = torch.empty(
            (self._num_blocks + 1, tokens, hidden), dtype=self.embed_tokens.weight.dtype, device=ids.device
        )
        ops.embedding(ids, self.embed_tokens.weight, out=bank_storage[0])
        mixed = torch.empty((tokens, hidden), dtype=bank_storage.dtype, device=ids.device)
        source_count = 1
        for block in range(self._num_blocks):
            partial: torch.Tensor | None = None
            bank = bank_storage[:source_count]
            first = block * self._layers_per_block
            last = first + self._layers_per_block - 1
            for index in range(first, last + 1):
                partial = self.layers.op_list[index].forward(
                    bank, partial, self._rotary_emb, ctx.kv_cache, batch, mixed,
                    out=bank_storage[source_count] if index == last else None,
                )
            source_count += 1
        return bank_storage[:source_count], mixed

    def forward(self) -> torch.Tensor:
        bank, mixed = self._trunk()
        return mix_and_norm(self.final_attn_res_mixer, self.norm, bank, None, mixed, bank.shape[0] - 1)


class MiniMindIMEForCausalLM(Qwen3ForCausalLM):
    """Standard-residual bundles use the Qwen3 decoder; ``block_attnres`` bundles
    use the Block AttnRes trunk with the same attention, RoPE, SwiGLU, KV-cache
    and LM-head formats."""

    def __init__(self, config: ModelConfig) -> None:
        if config.residual_type == "standard":
            super().__init__(config)
            return
        self.model = MiniMindBlockAttnResModel(config)
        self.attn_backend = self.model.attn_backend
        self.lm_head = LMHead(
            config.vocab_size,
            config.hidden_size,
            tie_word_embeddings=config.tie_word_embeddings,
            tied_embedding=self.model.embed_tokens if config.tie_word_embeddings else None,
        )

    def forward(self) -> torch.Tensor:
        if isinstance(self.model, MiniMindBlockAttnResModel):
            norm = self.model.norm
            return self.lm_head.forward_normed(self.model.forward_hidden(), None, norm.weight, norm.eps)
        return super().forward()
