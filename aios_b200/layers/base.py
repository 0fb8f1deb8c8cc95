"""Parameter tree (aios/layers/base.py:19-108).

Public tensor attributes are parameters, named by their attribute path; private
``_``-prefixed attributes are runtime state. The naming scheme must equal the
reference's so checkpoints and seeded synthetic weights map one to one.
"""

from __future__ import annotations

from abc import abstractmethod
from typing import Any, Dict, Generic, List, TypeAlias, TypeVar

import torch

_STATE_DICT: TypeAlias = Dict[str, torch.Tensor]


def _concat_prefix(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


class BaseOP:
    @abstractmethod
    def forward(self, *args: Any, **kwargs: Any) -> Any: ...

    def state_dict(self, *, prefix: str = "") -> _STATE_DICT:
        result: _STATE_DICT = {}
        for name, value in self.__dict__.items():
            if name.startswith("_"):
                continue
            key = _concat_prefix(prefix, name)
            if isinstance(value, torch.Tensor):
                result[key] = value
            elif isinstance(value, BaseOP):
                result.update(value.state_dict(prefix=key))
        return result

    def load_state_dict(self, state_dict: _STATE_DICT, *, prefix: str = "", _internal: bool = False) -> None:
        for name, value in list(self.__dict__.items()):
            if name.startswith("_"):
                continue
            key = _concat_prefix(prefix, name)
            if isinstance(value, torch.Tensor):
                item = state_dict.pop(key)
                assert isinstance(item, torch.Tensor)
                assert value.shape == item.shape, f"Shape mismatch for {key}: expected {value.shape}, got {item.shape}"
                setattr(self, name, item)
            elif isinstance(value, BaseOP):
                value.load_state_dict(state_dict, prefix=key, _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"Unexpected keys in state_dict: {list(state_dict.keys())}")
        self.on_weights_loaded()

    def on_weights_loaded(self) -> None:
        """Hook for ops that derive device-side data (packed weights) from parameters."""


class StateLessOP(BaseOP):
    def load_state_dict(self, state_dict: _STATE_DICT, *, prefix: str = "", _internal: bool = False) -> None:
        if not _internal and state_dict:
            raise RuntimeError(f"Unexpected keys in state_dict: {list(state_dict.keys())}")

    def state_dict(self, *, prefix: str = "") -> _STATE_DICT:
        return {}


T = TypeVar("T", bound=BaseOP)


class OPList(BaseOP, Generic[T]):
    def __init__(self, ops: List[T]):
        self.op_list = ops

    def state_dict(self, *, prefix: str = "") -> _STATE_DICT:
        result: _STATE_DICT = {}
        for i, op in enumerate(self.op_list):
            result.update(op.state_dict(prefix=_concat_prefix(prefix, str(i))))
        return result

    def load_state_dict(self, state_dict: _STATE_DICT, *, prefix: str = "", _internal: bool = False) -> None:
        for i, op in enumerate(self.op_list):
            op.load_state_dict(state_dict, prefix=_concat_prefix(prefix, str(i)), _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"Unexpected keys in state_dict: {list(state_dict.keys())}")
