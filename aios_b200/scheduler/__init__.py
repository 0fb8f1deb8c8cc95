from .cache import CacheManager
from .decode import DecodeManager
from .prefill import PrefillManager
from .scheduler import Scheduler
from .table import TableManager

__all__ = ["CacheManager", "DecodeManager", "PrefillManager", "Scheduler", "TableManager"]
