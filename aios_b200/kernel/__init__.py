"""B200 kernels behind the reference's kernel entry points (aios/kernel/__init__.py)."""

from .ops import b200_attnres_mix, store_cache

__all__ = ["store_cache", "b200_attnres_mix"]
