from __future__ import annotations

from abc import ABC, abstractmethod

import torch

from ..layers import BaseOP


class BaseLLMModel(ABC, BaseOP):
    @abstractmethod
    def forward(self) -> torch.Tensor: ...
