from .batcher import ContinuousBatcher
from .cache import CacheManager

__all__ = ["CacheManager", "ContinuousBatcher"]
