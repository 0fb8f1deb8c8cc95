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
from typing import List, Literal

import torch

from .core import Context, SamplingParams, reset_global_ctx, set_global_ctx
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
        if backend is not None:  # validated by ModelConfig: any reference name runs the sm_100a mixer
            config = replace(config, attnres_backend=str(backend))
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

    @torch.no_grad()
    def generate(
        self,
        prompts: List[str] | List[List[int]],
        sampling_params: SamplingParams | List[SamplingParams] | None = None,
        max_running_reqs: int | None = None,
        prefill_token_budget: int | None = None,
        debug_scheduler: bool = False,
        prompt_mode: Literal["chat", "raw"] = "chat",
        add_bos: bool = True,
    ) -> List[dict]:
        """Generates requests with continuous batching and varlen prefill
        (aios/llm/llm.py:98-175) on the same kernels as the IME path: prefill-first
        scheduling, one decode token per running request per step, KV slots
        (page_size 1) freed as soon as a request finishes. Returns one dict per
        prompt, in prompt order: uid, token_ids, text."""
        from .engine.engine import Engine
        from .scheduler.batcher import ContinuousBatcher

        if self.page_size != 1:
            raise ValueError("generate uses page_size 1 KV slots (build the LLM with page_size=1)")
        if sampling_params is None:
            sampling_params = SamplingParams()
        params_list = [sampling_params] * len(prompts) if isinstance(sampling_params, SamplingParams) else sampling_params
        if len(params_list) != len(prompts):
            raise ValueError("one SamplingParams per prompt")
        vocab = self.config.vocab_size
        for sp in params_list:  # the sampler's sort limit, checked before any KV is taken
            k = min(sp.top_k, vocab) if sp.top_k > 0 else (vocab if sp.top_p < 1.0 else 0)
            if not sp.is_greedy and k > 2048 and vocab > 16384:
                raise ValueError(f"sample: a sorted candidate set of {k} needs a vocabulary of at most 16384")
        all_ids: List[torch.Tensor] = []
        for prompt in prompts:
            if isinstance(prompt, str):
                if prompt_mode == "chat":
                    if not hasattr(self.tokenizer, "apply_chat_template"):
                        raise ValueError("chat prompts need a tokenizer with a chat template; use prompt_mode='raw'")
                    text = self.tokenizer.apply_chat_template([{"role": "user", "content": prompt}], tokenize=False,
                                                              add_generation_prompt=True, enable_thinking=False)
                    ids = torch.tensor(self.tokenizer.encode(text), dtype=torch.long)
                elif prompt_mode == "raw":
                    token_ids = self.tokenizer.encode(prompt, add_special_tokens=False)
                    if add_bos and self.tokenizer.bos_token_id is not None:
                        token_ids = [self.tokenizer.bos_token_id, *token_ids]
                    ids = torch.tensor(token_ids, dtype=torch.long)
                else:
                    raise ValueError(f"Unsupported prompt_mode: {prompt_mode}")
            else:
                ids = torch.tensor(prompt, dtype=torch.long)
            all_ids.append(ids)
        if not all_ids:
            return []
        # the decode attention kernel takes rows * (q heads per KV head) <= 64
        row_limit = max(1, 64 // (self.config.num_qo_heads // self.config.num_kv_heads))
        if max_running_reqs is None:
            max_running_reqs = len(prompts)
        max_running_reqs = max(1, min(max_running_reqs, len(prompts), row_limit))
        max_total_len = max(len(ids) + sp.max_tokens for ids, sp in zip(all_ids, params_list))
        if max_total_len > self.config.max_position_embeddings:
            raise ValueError(f"prompt + max_tokens exceeds the context: {max_total_len}")
        page_table = torch.zeros((max_running_reqs, max_total_len), dtype=torch.int32, device=self.device)
        saved_table = self.ctx.page_table
        self.ctx.page_table = page_table
        try:
            batcher = ContinuousBatcher(cache_manager=self.cache_manager, page_table=page_table,
                                        eos_token_id=self.tokenizer.eos_token_id, device=self.device,
                                        max_running=max_running_reqs, attn_backend=self.model.attn_backend,
                                        prefill_token_budget=prefill_token_budget)
            engine = Engine(model=self.model, mha_kv_cache=self.mha_kv_cache)
            for ids, sp in zip(all_ids, params_list):
                batcher.add_request(ids, sp)
            iteration = 0
            while batcher.has_work:
                batch = batcher.next_batch()
                if batch is None:
                    raise RuntimeError("generate: pending requests do not fit the KV cache")
                batcher.commit(batch, engine.run_batch(batch))
                if debug_scheduler:
                    print(f"[{iteration}] {batcher.describe(batch)}")
                iteration += 1
            return batcher.results(self.tokenizer)
        finally:
            self.ctx.page_table = saved_table
