from .base import BaseLLMModel
from .config import ModelConfig
from .weight import init_synthetic_weights, load_weights


def create_model(model_path: str, config: ModelConfig) -> BaseLLMModel:
    """aios/models/__init__.py:6-17: pick the model class from config or path."""
    name = model_path.lower()
    if config.model_type == "qwen3" or "qwen3" in name:
        from .qwen3 import Qwen3ForCausalLM

        return Qwen3ForCausalLM(config)
    if config.model_type == "minimind_ime_v3" or "minimind-ime" in name:
        from .minimind_ime import MiniMindIMEForCausalLM

        return MiniMindIMEForCausalLM(config)
    raise ValueError(f"Unsupported model: {model_path}")


__all__ = ["BaseLLMModel", "ModelConfig", "create_model", "load_weights", "init_synthetic_weights"]
