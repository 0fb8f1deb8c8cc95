"""Oracle restatement of the model forward (TEST INFRASTRUCTURE ONLY).

CPU torch forward of the standard-residual decoder (aios/models/qwen3.py:31-173)
and of the Block AttnRes trunk (aios/models/minimind_ime.py:193-354) over an
explicit slot-addressed KV cache (the MHAKVCache layout flattened to
[slots, Hkv, d], aios/kvcache/mha_pool.py:28-37).

``dtype=torch.float32`` is the pure-fp32 restatement (pinned against the
reference run in fp32); ``dtype=torch.bfloat16`` keeps bf16 storage between ops
with the reference's rounding points: every linear output, the norms, bf16 RoPE
arithmetic, the AttnRes weights and the residual adds. Matmuls accumulate in fp32
(``accumulate="fp32"``, as the reference's CPU run does), or in fp64
(``accumulate="fp64"``: every linear output is then the bf16 rounding of the
exact dot product). The two bf16 variants bound the rounding noise between
faithful implementations that differ only in summation order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops as oops


@dataclass
class Request:
    """One request of a forward: new tokens and where they live."""

    ids: list[int]
    positions: list[int]
    new_slots: list[int]  # KV slot of each new token
    key_slots: list[int]  # slot of every key position 0..max(positions)


class OracleModel:
    def __init__(self, config, state: dict[str, torch.Tensor], dtype: torch.dtype = torch.float32,
                 num_slots: int = 4096, mixer: str = "fused", accumulate: str = "fp32") -> None:
        self.cfg = config
        self.dtype = dtype
        if accumulate not in ("fp32", "fp64"):
            raise ValueError("accumulate must be 'fp32' or 'fp64'")
        self._acc = torch.float64 if accumulate == "fp64" else torch.float32
        self.w = {k: v.detach().to("cpu", dtype) for k, v in state.items()}
        self.hq, self.hkv, self.d = config.num_qo_heads, config.num_kv_heads, config.head_dim
        self.eps = config.rms_norm_eps
        self.scale = config.head_dim ** -0.5
        self.cos, self.sin = oops.rope_cache(config.head_dim, config.max_position_embeddings, config.rope_theta)
        L = config.num_layers
        self.k = torch.zeros((L, num_slots, self.hkv, self.d), dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.block = config.residual_type == "block_attnres"
        if mixer not in ("fused", "eager"):
            raise ValueError("mixer must be 'fused' (single rounding) or 'eager' (training semantics)")
        self.mixer = mixer
        self.wq = {}
        if self.block:
            for name in list(self.w):
                if name.endswith(".query"):
                    base = name[: -len(".query")]
                    self.wq[base] = state[name].float().cpu() * state[base + ".key_norm.weight"].float().cpu()

    # ---- building blocks -------------------------------------------------------
    def _linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return (x.to(self._acc) @ self.w[name].to(self._acc).T).float().to(self.dtype)

    def _attention(self, layer: int, prefix: str, x: torch.Tensor, reqs: list[Request]) -> torch.Tensor:
        hq, hkv, d = self.hq, self.hkv, self.d
        qkv = self._linear(x, f"{prefix}.self_attn.qkv_proj.weight")
        T = qkv.shape[0]
        q = qkv[:, : hq * d].reshape(T, hq, d)
        k = qkv[:, hq * d : (hq + hkv) * d].reshape(T, hkv, d)
        v = qkv[:, (hq + hkv) * d :].reshape(T, hkv, d)
        q = oops.rmsnorm(q, self.w[f"{prefix}.self_attn.q_norm.weight"], self.eps)
        k = oops.rmsnorm(k, self.w[f"{prefix}.self_attn.k_norm.weight"], self.eps)
        pos = torch.tensor([p for r in reqs for p in r.positions])
        q = oops.apply_rope(q, self.cos[pos], self.sin[pos])
        k = oops.apply_rope(k, self.cos[pos], self.sin[pos])
        slots = torch.tensor([s for r in reqs for s in r.new_slots])
        self.k[layer, slots] = k
        self.v[layer, slots] = v
        outs, t0 = [], 0
        for r in reqs:
            n = len(r.ids)
            ks = torch.tensor(r.key_slots)
            o = oops.attention(q[t0 : t0 + n], self.k[layer, ks], self.v[layer, ks], torch.tensor(r.positions),
                               self.scale)
            outs.append(o.to(self.dtype))
            t0 += n
        return torch.cat(outs).reshape(T, hq * d)

    def _mlp(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        gu = self._linear(x, f"{prefix}.mlp.gate_up_proj.weight")
        return self._linear(oops.silu_and_mul(gu), f"{prefix}.mlp.down_proj.weight")

    def _mix(self, base: str, bank: torch.Tensor, partial: torch.Tensor | None) -> torch.Tensor:
        fn = oops.attnres_mix_fused if self.mixer == "fused" else oops.attnres_mix_eager
        return fn(bank, partial, self.wq[base], self.eps)

    # ---- forward ----------------------------------------------------------------
    def forward(self, reqs: list[Request], all_logits: bool = False) -> torch.Tensor:
        """Logits of each request's last new token ([len(reqs), V]) or of every
        new token; KV of the new tokens is written into the cache."""
        ids = torch.tensor([t for r in reqs for t in r.ids])
        h = self.w["model.embed_tokens.weight"][ids]
        if self.block:
            h = self._forward_block(h, reqs)
        else:
            residual = None
            for layer in range(self.cfg.num_layers):
                p = f"model.layers.{layer}"
                if residual is None:
                    x, residual = oops.rmsnorm(h, self.w[f"{p}.input_layernorm.weight"], self.eps), h
                else:
                    x, residual = oops.fused_add_rmsnorm(h, residual, self.w[f"{p}.input_layernorm.weight"], self.eps)
                a = self._linear(self._attention(layer, p, x, reqs), f"{p}.self_attn.o_proj.weight")
                x, residual = oops.fused_add_rmsnorm(a, residual, self.w[f"{p}.post_attention_layernorm.weight"],
                                                     self.eps)
                h = self._mlp(p, x)
            h, _ = oops.fused_add_rmsnorm(h, residual, self.w["model.norm.weight"], self.eps)
        if not all_logits:
            last, acc = [], 0
            for r in reqs:
                acc += len(r.ids)
                last.append(acc - 1)
            h = h[torch.tensor(last)]
        return self._linear(h, "model.embed_tokens.weight")

    def _forward_block(self, h: torch.Tensor, reqs: list[Request]) -> torch.Tensor:
        cfg = self.cfg
        per = cfg.num_layers // cfg.attnres_num_blocks
        bank = [h]
        for b in range(cfg.attnres_num_blocks):
            partial = None
            src = torch.stack(bank)
            for layer in range(b * per, (b + 1) * per):
                p = f"model.layers.{layer}"
                hidden = self._mix(f"{p}.attn_res_mixer", src, partial)
                x = oops.rmsnorm(hidden, self.w[f"{p}.input_layernorm.weight"], self.eps)
                delta = self._linear(self._attention(layer, p, x, reqs), f"{p}.self_attn.o_proj.weight")
                partial = delta if partial is None else (partial.float() + delta.float()).to(self.dtype)
                hidden = self._mix(f"{p}.mlp_res_mixer", src, partial)
                x = oops.rmsnorm(hidden, self.w[f"{p}.post_attention_layernorm.weight"], self.eps)
                partial = (partial.float() + self._mlp(p, x).float()).to(self.dtype)
            bank.append(partial)
        hidden = self._mix("model.final_attn_res_mixer", torch.stack(bank), None)
        return oops.rmsnorm(hidden, self.w["model.norm.weight"], self.eps)
