from .sample import Sampler, stateless_uniforms

__all__ = ["Sampler", "stateless_uniforms"]
