"""LLM facade (replaces aios/llm/llm.py:26-96, the wiring part).

``LLM(model_path, ...)`` loads an HF/safetensors MiniMind-IME or Qwen3 bundle;
``LLM(config=ModelConfig(...), seed=0)`` (or ``shape="S10"``) builds the model with
the seeded synthetic weights the benchmarks use, plus the synthetic tokenizer.
Both end with the same objects the IME engine reads: ``model``, ``tokenizer``,
``ctx``, ``cache_manager``, ``num_pages``, ``config``, ``device``.

KV pool: ``page_size`` 1 (the reference's layout; slot ids then equal the
reference's bit for bit) or 16 (16-token pages). ``num_pages`` may be given
directly; otherwise ``kv_cache_max_tokens`` / free memory decide, as in
aios/llm/llm.py:77-96. The newest LLM owns the process-global context.
"""

from __future__ import annotations

import os
from dataclasses import replace

import torch

from .core import Context, reset_global_ctx, set_global_ctx
from .kvcache import MHAKVCache
from .models import ModelConfig, create_model, init_synthetic_weights, load_weights
from .models.shapes import shape as named_shape
from .scheduler import CacheManager
from .tokenizer import SyntheticTokenizer


class LLM:
    def __init__(self, model_path: str | None = None, dtype: torch.dtype = torch.bfloat16, **kwargs):
        self.device = torch.device(kwargs.get("device", "cuda"))
        if self.device.type != "cuda":
            raise ValueError("aios_b200 runs on CUDA (sm_100a) devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        torch.cuda.set_device(self.device)
        if dtype != torch.bfloat16:
            raise ValueError("aios_b200 serves bf16 models")
        self.dtype = dtype
        config = kwargs.get("config")
        if config is None and kwargs.get("shape") is not None:
            config = named_shape(kwargs["shape"])
        synthetic = model_path is None
        if synthetic:
            if config is None:
                raise ValueError("pass model_path, config= or shape=")
        else:
            config = self._load_config(model_path)
        backend = kwargs.get("attnres_backend")
        if backend is not None and str(backend) != "b200":
            raise ValueError("attnres_backend must be 'b200' (the sm_100a fused mixer)")
        config = replace(config, attnres_backend="b200")
        self.config = config
        self._num_layers = config.num_layers
        with torch.device("meta"):
            self.model = create_model(model_path or "minimind-ime", config)
        workspace = kwargs.get("attention_workspace_size")
        if workspace is not None:
            if workspace <= 0:
                raise ValueError("attention_workspace_size must be positive")
            self.model.attn_backend.workspace_size = int(workspace)
        if synthetic:
            init_synthetic_weights(self.model, self.device, dtype, seed=int(kwargs.get("seed", 0)))
            self.tokenizer = kwargs.get("tokenizer") or SyntheticTokenizer(config.vocab_size)
        else:
            load_weights(self.model, model_path, self.device, dtype)
            from transformers import AutoTokenizer

            self.tokenizer = kwargs.get("tokenizer") or AutoTokenizer.from_pretrained(model_path)
        self.model.model._rotary_emb.set_device(self.device)
        self.page_size = int(kwargs.get("page_size", 1))
        self.num_pages = self._determine_num_pages(
            config, kwargs.get("memory_ratio", 0.9), kwargs.get("kv_cache_max_tokens"), kwargs.get("num_pages")
        )
        self.mha_kv_cache = MHAKVCache(
            num_kv_heads=config.num_kv_heads, num_layers=config.num_layers, head_dim=config.head_dim,
            num_pages=self.num_pages, page_size=self.page_size, dtype=dtype, device=self.device,
        )
        self.cache_manager = CacheManager(self.device, self.num_pages, self.page_size)
        self.ctx = Context(page_size=self.page_size)
        self.ctx.kv_cache = self.mha_kv_cache
        self.ctx.attn_backend = self.model.attn_backend
        self.ctx.page_table = torch.zeros((1, config.max_position_embeddings), dtype=torch.int32, device=self.device)
        reset_global_ctx()
        set_global_ctx(self.ctx)

    @staticmethod
    def _load_config(model_path: str) -> ModelConfig:
        if not os.path.isdir(model_path):
            raise FileNotFoundError(f"model directory not found: {model_path} (no network downloads)")
        try:
            from transformers import AutoConfig

            return ModelConfig.from_hf(AutoConfig.from_pretrained(model_path))
        except (ValueError, OSError, KeyError, AttributeError):
            return ModelConfig.from_json(model_path)

    def _determine_num_pages(self, config: ModelConfig, memory_ratio: float, max_tokens, num_pages) -> int:
        if num_pages is not None:
            if int(num_pages) <= 1:
                raise ValueError("num_pages must be greater than 1")
            return int(num_pages)
        torch.cuda.synchronize(self.device)
        free_memory = torch.cuda.mem_get_info(self.device)[0]
        per_page = 2 * config.head_dim * config.num_kv_heads * self.page_size * 2 * config.num_layers
        pages = int(memory_ratio * free_memory) // per_page
        if max_tokens is not None:
            if max_tokens <= 1:
                raise ValueError("kv_cache_max_tokens must be greater than 1")
            pages = min(pages, max(1, int(max_tokens) // self.page_size))
        if pages <= 1:
            raise RuntimeError(f"Not enough GPU memory for KV cache (free={free_memory}, per_page={per_page})")
        return pages
