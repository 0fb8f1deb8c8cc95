from .b200 import B200AttentionBackend, B200AttentionMetadata
from .base import BaseAttentionBackend, BaseAttentionMetadata, HybridAttentionBackend

__all__ = [
    "BaseAttentionBackend",
    "BaseAttentionMetadata",
    "HybridAttentionBackend",
    "B200AttentionBackend",
    "B200AttentionMetadata",
]
