from .base import BaseKVCache
from .mha_pool import MHAKVCache

__all__ = ["BaseKVCache", "MHAKVCache"]
