from .activation import silu_and_mul
from .base import BaseOP, OPList, StateLessOP, _concat_prefix
from .embedding import Embedding, LMHead
from .linear import Linear, LinearColParallelMerged, LinearQKVMerged
from .norm import RMSNorm, RMSNormFused
from .rotary import RotaryEmbedding

__all__ = [
    "silu_and_mul",
    "BaseOP", "StateLessOP", "OPList", "_concat_prefix",
    "Linear", "LinearColParallelMerged", "LinearQKVMerged",
    "RMSNorm", "RMSNormFused", "RotaryEmbedding",
    "Embedding", "LMHead",
]
