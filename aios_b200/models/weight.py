"""Weights: safetensors loading with projection packing (aios/models/weight.py:14-70)
and the seeded synthetic initialisation used for benchmarks and parity runs.
"""

from __future__ import annotations

import glob
import os
from collections.abc import Iterable

import torch

from ..layers import BaseOP

# HF checkpoints keep these projections separate; the fused operators consume
# them concatenated along the output dimension.
packed_modules_mapping: dict[str, tuple[str, ...]] = {
    "qkv_proj": ("q_proj", "k_proj", "v_proj"),
    "gate_up_proj": ("gate_proj", "up_proj"),
}


def _checkpoint_index(files: Iterable[str]) -> dict[str, str]:
    import safetensors

    index: dict[str, str] = {}
    for path in files:
        with safetensors.safe_open(path, framework="pt", device="cpu") as handle:
            for name in handle.keys():
                if name in index:
                    raise RuntimeError(f"Duplicate safetensors key: {name}")
                index[name] = path
    return index


def _read_tensor(index: dict[str, str], name: str) -> torch.Tensor:
    import safetensors

    try:
        path = index[name]
    except KeyError as exc:
        raise KeyError(f"Checkpoint is missing required tensor: {name}") from exc
    with safetensors.safe_open(path, framework="pt", device="cpu") as handle:
        return handle.get_tensor(name)


def _packed_source_names(target_name: str) -> tuple[str, ...] | None:
    for packed_name, source_names in packed_modules_mapping.items():
        marker = f".{packed_name}."
        if marker in target_name:
            return tuple(target_name.replace(marker, f".{src}.") for src in source_names)
    return None


def load_weights(model: BaseOP, model_path: str, device: torch.device, dtype: torch.dtype) -> None:
    """Load an HF safetensors checkpoint, packing qkv and gate/up projections."""
    files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"No .safetensors files found in {model_path}")
    index = _checkpoint_index(files)
    fused: dict[str, torch.Tensor] = {}
    for target in model.state_dict():
        sources = _packed_source_names(target)
        if sources is None:
            tensor = _read_tensor(index, target)
        else:
            tensor = torch.cat([_read_tensor(index, name) for name in sources], dim=0)
        fused[target] = tensor.to(device=device, dtype=dtype)
    model.load_state_dict(fused)


def synthetic_state_dict(model: BaseOP, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded random weights in the benchmark protocol's rule: walk the state dict
    in insertion order with one generator; ``*norm.weight`` = 1, everything else
    (including AttnRes queries) ~ N(0, 1) * std. Returns fp32 CPU tensors."""
    gen = torch.Generator().manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, param in model.state_dict().items():
        shape = tuple(param.shape)
        if name.endswith("norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.float32)
        else:
            out[name] = torch.randn(shape, generator=gen, dtype=torch.float32) * std
    return out


def init_synthetic_weights(
    model: BaseOP, device: torch.device, dtype: torch.dtype = torch.bfloat16, seed: int = 0, std: float = 0.02
) -> None:
    state = {k: v.to(device=device, dtype=dtype) for k, v in synthetic_state_dict(model, seed, std).items()}
    model.load_state_dict(state)
