"""Model configuration (aios/models/config.py:8-113) plus the ``b200`` AttnRes backend.

The AttnRes backend slot accepts the reference's four names (``reference``,
``eager``, ``compiled``, ``triton``; aios/models/config.py:27,34-40) and ``b200``.
This build has one mixer, the sm_100a kernel, so every accepted name runs it; the
name is kept as given so that a reference config round-trips unchanged. Any other
name raises the reference's ``ValueError``.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass

# reference names (all served by the one sm_100a mixer) plus this build's own
ATTNRES_BACKENDS = frozenset({"reference", "eager", "compiled", "triton", "b200"})


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    hidden_size: int
    vocab_size: int
    intermediate_size: int
    hidden_act: str
    rms_norm_eps: float
    rope_theta: float
    max_position_embeddings: int
    tie_word_embeddings: bool
    model_type: str = "unknown"
    architecture_revision: str = ""
    residual_type: str = "standard"
    attnres_num_blocks: int = 0
    attnres_alpha: float = 1.0
    attnres_backend: str = "triton"  # the reference's default name; runs the sm_100a mixer

    def __post_init__(self) -> None:
        if self.residual_type not in {"standard", "block_attnres"}:
            raise ValueError("residual_type must be 'standard' or 'block_attnres'")
        if self.attnres_backend not in ATTNRES_BACKENDS:
            raise ValueError("attnres_backend must be 'reference', 'eager', 'compiled', 'triton' or 'b200' "
                             "(all run the sm_100a fused mixer)")
        if self.residual_type == "block_attnres":
            if self.attnres_num_blocks < 1:
                raise ValueError("block_attnres requires attnres_num_blocks >= 1")
            if self.num_layers % self.attnres_num_blocks:
                raise ValueError("num_layers must be divisible by attnres_num_blocks")
            if float(self.attnres_alpha) != 1.0:
                raise ValueError("AIOS only serves fully migrated Block AttnRes snapshots with attnres_alpha=1.0")

    @property
    def layers_per_attnres_block(self) -> int:
        if self.residual_type != "block_attnres":
            raise ValueError("standard residual models do not have AttnRes blocks")
        return self.num_layers // self.attnres_num_blocks

    @classmethod
    def _from_mapping(cls, get) -> ModelConfig:
        hidden = get("hidden_size")
        heads = get("num_attention_heads")
        return cls(
            num_layers=get("num_hidden_layers"),
            num_qo_heads=heads,
            num_kv_heads=get("num_key_value_heads", heads),
            head_dim=get("head_dim", hidden // heads),
            hidden_size=hidden,
            vocab_size=get("vocab_size"),
            intermediate_size=get("intermediate_size"),
            hidden_act=get("hidden_act", "silu"),
            rms_norm_eps=get("rms_norm_eps", 1e-6),
            rope_theta=get("rope_theta", 1000000.0),
            max_position_embeddings=get("max_position_embeddings", 32768),
            tie_word_embeddings=get("tie_word_embeddings", False),
            model_type=get("model_type", "unknown"),
            architecture_revision=get("architecture_revision", ""),
            residual_type=get("residual_type", "standard"),
            attnres_num_blocks=get("attnres_num_blocks", 0),
            attnres_alpha=get("attnres_alpha", 1.0),
        )

    @classmethod
    def from_hf(cls, config) -> ModelConfig:
        missing = object()

        def get(name, default=missing):
            value = getattr(config, name, missing)
            if value is missing or value is None:
                if default is missing:
                    raise AttributeError(name)
                return default
            return value

        return cls._from_mapping(get)

    @classmethod
    def from_json(cls, model_path: str) -> ModelConfig:
        with open(os.path.join(model_path, "config.json")) as f:
            data = json.load(f)
        missing = object()

        def get(name, default=missing):
            if name in data:
                return data[name]
            if default is missing:
                raise KeyError(name)
            return default

        return cls._from_mapping(get)
