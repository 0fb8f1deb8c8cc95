from .cache import CacheManager

__all__ = ["CacheManager"]
