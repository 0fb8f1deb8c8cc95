from .engine import Engine
from .sample import Sampler, stateless_uniforms

__all__ = ["Engine", "Sampler", "stateless_uniforms"]
