"""The model shapes the CandidateGroup path is built and measured on.

* S06 — the 0.06B standard-residual shape as the benchmark spec states it:
  8 layers, hidden 768, 8 query / 2 KV heads of 96, FFN 2048, vocab 6400.
* S10 — the 0.1B MiniMind-IME shape documented by the reference (14 layers,
  12 query / 4 KV heads of 64, vocab 16384, 100,687,360 parameters).
* S10L — S06's dims with 14 layers.
* S21 — the 0.214B Block AttnRes shape: S10 dims, 32 layers in 8 blocks.
All use RoPE theta 1e6, RMSNorm eps 1e-6, tied embeddings, 512 positions.
"""

from __future__ import annotations

from dataclasses import replace

from .config import ModelConfig

_BASE = dict(
    hidden_size=768,
    intermediate_size=2048,
    hidden_act="silu",
    rms_norm_eps=1e-6,
    rope_theta=1e6,
    max_position_embeddings=512,
    tie_word_embeddings=True,
    model_type="minimind_ime_v3",
)

S06 = ModelConfig(num_layers=8, num_qo_heads=8, num_kv_heads=2, head_dim=96, vocab_size=6400,
                  architecture_revision="s06", **_BASE)
S10 = ModelConfig(num_layers=14, num_qo_heads=12, num_kv_heads=4, head_dim=64, vocab_size=16384,
                  architecture_revision="s10", **_BASE)
S10L = replace(S06, num_layers=14, architecture_revision="s10l")
S21 = replace(S10, num_layers=32, residual_type="block_attnres", attnres_num_blocks=8, architecture_revision="s21")

SHAPES = {"S06": S06, "S10": S10, "S10L": S10L, "S21": S21}


def shape(name: str) -> ModelConfig:
    try:
        return SHAPES[name.upper()]
    except KeyError as exc:
        raise ValueError(f"unknown model shape {name!r}; choose from {sorted(SHAPES)}") from exc
