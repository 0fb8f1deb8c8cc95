"""Checkpoint loading (aios/models/weight.py:14-70, aios/models/config.py) on the
CPU: a synthetic checkpoint in the Hugging Face layout (separate q/k/v and
gate/up projections, config.json) is read back into the packed model exactly."""

from __future__ import annotations

import dataclasses
import json

import pytest
import torch

from aios_b200.models import shapes
from aios_b200.models.config import ModelConfig
from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM
from aios_b200.models.weight import load_weights, synthetic_state_dict


def _hf_tensors(cfg, state: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    q = cfg.num_qo_heads * cfg.head_dim
    kv = cfg.num_kv_heads * cfg.head_dim
    out = {}
    for name, t in state.items():
        t = t.to(torch.bfloat16).contiguous()
        if ".qkv_proj." in name:
            for part, piece in zip(("q_proj", "k_proj", "v_proj"), torch.split(t, [q, kv, kv])):
                out[name.replace(".qkv_proj.", f".{part}.")] = piece.contiguous()
        elif ".gate_up_proj." in name:
            for part, piece in zip(("gate_proj", "up_proj"), torch.chunk(t, 2)):
                out[name.replace(".gate_up_proj.", f".{part}.")] = piece.contiguous()
        else:
            out[name] = t
    return out


def _hf_config(cfg) -> dict:
    return {
        "hidden_size": cfg.hidden_size, "num_attention_heads": cfg.num_qo_heads,
        "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "num_hidden_layers": cfg.num_layers,
        "vocab_size": cfg.vocab_size, "intermediate_size": cfg.intermediate_size, "rms_norm_eps": cfg.rms_norm_eps,
        "rope_theta": cfg.rope_theta, "max_position_embeddings": cfg.max_position_embeddings,
        "tie_word_embeddings": cfg.tie_word_embeddings, "model_type": "minimind",
        "residual_type": cfg.residual_type, "attnres_num_blocks": cfg.attnres_num_blocks,
        "attnres_alpha": cfg.attnres_alpha,
    }


@pytest.mark.parametrize("cfg", [dataclasses.replace(shapes.S10, num_layers=2),
                                 dataclasses.replace(shapes.S21, num_layers=4, attnres_num_blocks=2)],
                         ids=["s10_l2", "s21_l4"])
def test_checkpoint_round_trip(tmp_path, cfg) -> None:
    from safetensors.torch import save_file

    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    state = synthetic_state_dict(meta, seed=5)
    tensors = _hf_tensors(cfg, state)
    # two shards, like a real multi-file checkpoint
    names = sorted(tensors)
    save_file({n: tensors[n] for n in names[::2]}, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({n: tensors[n] for n in names[1::2]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(_hf_config(cfg)))

    loaded_cfg = ModelConfig.from_json(str(tmp_path))
    for field in ("num_layers", "num_qo_heads", "num_kv_heads", "head_dim", "hidden_size", "vocab_size",
                  "intermediate_size", "residual_type", "attnres_num_blocks", "tie_word_embeddings"):
        assert getattr(loaded_cfg, field) == getattr(cfg, field), field

    with torch.device("meta"):
        model = MiniMindIMEForCausalLM(loaded_cfg)
    load_weights(model, str(tmp_path), torch.device("cpu"), torch.bfloat16)
    got = model.state_dict()
    assert set(got) == set(state)
    for name, want in state.items():
        assert torch.equal(got[name].cpu(), want.to(torch.bfloat16)), name


def test_checkpoint_missing_tensor_is_reported(tmp_path) -> None:
    from safetensors.torch import save_file

    cfg = dataclasses.replace(shapes.S10, num_layers=1)
    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    tensors = _hf_tensors(cfg, synthetic_state_dict(meta, seed=1))
    tensors.pop("model.layers.0.self_attn.k_proj.weight")
    save_file(tensors, str(tmp_path / "model.safetensors"))
    with torch.device("meta"):
        model = MiniMindIMEForCausalLM(cfg)
    with pytest.raises(KeyError, match="k_proj"):
        load_weights(model, str(tmp_path), torch.device("cpu"), torch.bfloat16)
