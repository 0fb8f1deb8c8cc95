"""The unmodified reference engine (7155/aios, Python) run on the CPU — TEST AND
BASELINE INFRASTRUCTURE ONLY.

The reference's keystroke path, ``ImeCompletionEngine.complete``
(aios/ime.py:415-640), is imported as-is from an installed copy of the reference
(``baseline/_ref``, made by ``pip install --target``; or a checkout's ``python/``
directory). Its GPU-only pieces are replaced by the smallest shims that let it
run on host cores, and nothing else is touched:

1. FlashInfer ``rmsnorm`` / ``fused_add_rmsnorm`` / ``silu_and_mul`` (imported
   lazily by aios/layers/norm.py:12,27 and aios/layers/activation.py:10) become
   torch expressions of the same arithmetic: fp32 math, one rounding to the
   storage dtype;
2. the attention backend becomes ``CpuBackend``: it stores K/V through the
   reference's own ``store_kv`` call shape and runs the reference's own
   ``_sdpa_prefill_attention`` (aios/attention/flashinfer.py:33-91) per request
   over the keys its page-table row lists, as ``_prefill_with_sdpa``
   (aios/attention/flashinfer.py:328-372) does for prefill and decode;
3. the KV cache becomes ``CpuKV``, the reference layout ``[2, L, P, 1, Hkv, d]``
   (aios/kvcache/mha_pool.py:28-32) in host memory;
4. ``torch.cuda.Event`` becomes a host-clock event.

The model weights follow the benchmark rule (state-dict order, one generator
seeded 0, ``*norm.weight`` = 1, everything else N(0, 1) * 0.02) and the tokenizer
maps ids >= 10 to single CJK characters (0 pad, 1 BOS, 2 EOS, 3-9 the terminal
punctuation), so the same seeded prefixes reach the same token ids as on the GPU.
This module imports nothing from the product package.
"""

from __future__ import annotations

import dataclasses
import importlib
import os
import sys
import time
import types
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[1]
DEFAULT_INSTALL = REPO / "baseline" / "_ref"

# Model shapes of the benchmark protocol, as reference ModelConfig fields.
_BASE = dict(num_layers=14, num_qo_heads=12, num_kv_heads=4, head_dim=64, hidden_size=768, vocab_size=16384,
             intermediate_size=2048, hidden_act="silu", rms_norm_eps=1e-6, rope_theta=1e6,
             max_position_embeddings=512, tie_word_embeddings=True, model_type="minimind_ime_v3")
SHAPES = {
    "S10": dict(_BASE, architecture_revision="s10"),
    "S06": dict(_BASE, num_layers=8, num_qo_heads=8, num_kv_heads=2, head_dim=96, vocab_size=6400,
                architecture_revision="s06"),
    "S10L": dict(_BASE, num_layers=14, num_qo_heads=8, num_kv_heads=2, head_dim=96, vocab_size=6400,
                 architecture_revision="s10l"),
    "S21": dict(_BASE, num_layers=32, residual_type="block_attnres", attnres_num_blocks=8,
                architecture_revision="s21"),
}

TERMINALS = "。！？；!?;"
_FIRST_CJK = 3 + len(TERMINALS)


class ShimTokenizer:
    """Ids <-> characters: 3..9 the terminal punctuation, >= 10 one CJK character
    each (U+4E00 upwards); decode(encode(s)) == s for such strings."""

    pad_token_id, bos_token_id, eos_token_id = 0, 1, 2

    def __init__(self, vocab_size: int) -> None:
        self.vocab_size = vocab_size

    def _char(self, i: int) -> str:
        if 3 <= i < _FIRST_CJK:
            return TERMINALS[i - 3]
        return chr(0x4E00 + i - _FIRST_CJK) if _FIRST_CJK <= i < self.vocab_size else ""

    def _id(self, ch: str):
        if ch in TERMINALS:
            return 3 + TERMINALS.index(ch)
        i = ord(ch) - 0x4E00 + _FIRST_CJK
        return i if _FIRST_CJK <= i < self.vocab_size else None

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [i for i in map(self._id, text) if i is not None]
        return [self.bos_token_id, *ids] if add_special_tokens else ids

    def decode(self, ids, skip_special_tokens: bool = True, **_) -> str:
        out = []
        for i in map(int, ids):
            if i < 3:
                if not skip_special_tokens:
                    out.append(("<pad>", "<s>", "</s>")[i])
                continue
            out.append(self._char(i))
        return "".join(out)

    def batch_decode(self, sequences, skip_special_tokens: bool = True, **_) -> list[str]:
        return [self.decode(s, skip_special_tokens) for s in sequences]

    def text_for(self, ids) -> str:
        return "".join(self._char(int(i)) for i in ids)


# ---- shim 1: FlashInfer norms / activation as torch expressions -------------
def fi_rmsnorm(x, w, eps, out=None, **_):
    xf = x.float()
    y = (xf * (1.0 / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps)) * w.float()).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def fi_fused_add_rmsnorm(x, residual, w, eps, **_):
    s = x.float() + residual.float()
    residual.copy_(s.to(residual.dtype))
    x.copy_((s * (1.0 / torch.sqrt((s * s).mean(-1, keepdim=True) + eps)) * w.float()).to(x.dtype))


def fi_silu_and_mul(x, out=None, **_):
    f = x.shape[-1] // 2
    g, u = x[..., :f].float(), x[..., f:].float()
    y = (g / (1.0 + torch.exp(-g)) * u).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


# ---- shim 4: host-clock CUDA event -------------------------------------------
class HostEvent:
    def __init__(self, *a, **k):
        self.t = 0.0

    def record(self, *a, **k):
        self.t = time.perf_counter()

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return (other.t - self.t) * 1e3


def install(reference: str | os.PathLike | None = None) -> types.SimpleNamespace:
    """Imports the reference package from `reference` (default: the installed copy
    under baseline/_ref, or $AIOS_REFERENCE) with the four shims in place, and
    returns the modules the runner uses."""
    path = Path(reference or os.environ.get("AIOS_REFERENCE") or DEFAULT_INSTALL)
    if not (path / "aios" / "ime.py").exists():
        raise FileNotFoundError(f"no reference package (aios/ime.py) under {path}")
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    try:
        import flashinfer
    except ImportError:  # the shims are all the reference calls of it on this path
        flashinfer = types.ModuleType("flashinfer")
        sys.modules["flashinfer"] = flashinfer
    flashinfer.rmsnorm = fi_rmsnorm
    flashinfer.fused_add_rmsnorm = fi_fused_add_rmsnorm
    flashinfer.silu_and_mul = fi_silu_and_mul
    torch.cuda.Event = HostEvent
    mods = types.SimpleNamespace()
    mods.core = importlib.import_module("aios.core")
    mods.attn_base = importlib.import_module("aios.attention.base")
    mods.attn_fi = importlib.import_module("aios.attention.flashinfer")
    mods.sample = importlib.import_module("aios.engine.sample")
    mods.ime = importlib.import_module("aios.ime")
    mods.config = importlib.import_module("aios.models.config")
    mods.minimind = importlib.import_module("aios.models.minimind_ime")
    mods.cache = importlib.import_module("aios.scheduler.cache")
    if not Path(mods.ime.__file__).resolve().is_relative_to(path.resolve()):
        raise RuntimeError(f"aios was imported from {mods.ime.__file__}, not from {path}")
    return mods


def make_backend_classes(mods):
    """Shims 2 and 3 against the reference's own base classes."""
    BaseAttentionBackend = mods.attn_base.BaseAttentionBackend
    BaseAttentionMetadata = mods.attn_base.BaseAttentionMetadata
    sdpa = mods.attn_fi._sdpa_prefill_attention
    core = mods.core

    @dataclasses.dataclass
    class CpuMeta(BaseAttentionMetadata):
        cu: torch.Tensor

        def get_last_indices(self, bs):
            return self.cu[1 : 1 + bs].long() - 1

    class CpuBackend(BaseAttentionBackend):
        def __init__(self, config):
            self.hkv, self.d = config.num_kv_heads, config.head_dim
            self.scale = config.head_dim**-0.5

        def prepare_metadata(self, batch):
            cu = torch.tensor([0] + [r.extend_len for r in batch.reqs]).cumsum(0)
            batch.attn_metadata = CpuMeta(cu=cu)
            return batch.attn_metadata

        def forward(self, q, k, v, kv, layer, batch):
            ctx = core.get_global_ctx()
            kv.store_kv(k, v, batch.out_loc.view(-1), layer)
            kc = kv.k_cache(layer).view(-1, self.hkv, self.d)
            vc = kv.v_cache(layer).view(-1, self.hkv, self.d)
            outs, off = [], 0
            for req in batch.reqs:
                n = req.extend_len
                idx = ctx.page_table[req.table_idx, : req.device_len].long()
                outs.append(sdpa(q[off : off + n], kc[idx], vc[idx], cached_len=req.cached_len, sm_scale=self.scale))
                off += n
            return torch.cat(outs).reshape(q.shape[0], -1)

    class CpuKV:
        def __init__(self, layers, pages, hkv, d, dtype):
            self.buf = torch.zeros((2, layers, pages, 1, hkv, d), dtype=dtype)
            self._shape = (pages, hkv, d)

        def k_cache(self, i):
            return self.buf[0, i]

        def v_cache(self, i):
            return self.buf[1, i]

        def store_kv(self, k, v, loc, layer):
            self.buf[0, layer].view(self._shape)[loc.long()] = k
            self.buf[1, layer].view(self._shape)[loc.long()] = v

        @property
        def dtype(self):
            return self.buf.dtype

    return CpuBackend, CpuKV


def synthetic_weights(model, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """The benchmark weight rule: state-dict order, one generator, norms = 1."""
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for name, param in model.state_dict().items():
        shape = tuple(param.shape)
        out[name] = (torch.ones(shape) if name.endswith("norm.weight")
                     else torch.randn(shape, generator=gen, dtype=torch.float32) * std)
    return out


def build_llm(mods, config_fields: dict, num_pages: int, dtype=torch.float32, state: dict | None = None,
              tokenizer=None) -> types.SimpleNamespace:
    """A duck-typed ``llm`` for the reference engine: the reference model (eager
    AttnRes backend) with CPU attention and KV shims, the reference CacheManager
    over `num_pages` one-token pages, and the shim tokenizer."""
    CpuBackend, CpuKV = make_backend_classes(mods)
    rcfg = mods.config.ModelConfig(**{**config_fields, "attnres_backend": "eager"})
    with torch.device("meta"):
        model = mods.minimind.MiniMindIMEForCausalLM(rcfg)
    if state is None:
        state = synthetic_weights(model)
    model.load_state_dict({k: v.to(dtype) for k, v in state.items()})
    model.model._rotary_emb.set_device(torch.device("cpu"))
    backend = CpuBackend(rcfg)
    model.attn_backend = backend
    model.model.attn_backend = backend
    for layer in model.model.layers.op_list:
        layer.self_attn._attn_backend = backend
    mods.core._GLOBAL_CTX = None
    ctx = mods.core.Context(page_size=1)
    ctx.kv_cache = CpuKV(rcfg.num_layers, num_pages, rcfg.num_kv_heads, rcfg.head_dim, dtype)
    ctx.attn_backend = backend
    mods.core.set_global_ctx(ctx)
    return types.SimpleNamespace(
        model=model, tokenizer=tokenizer or ShimTokenizer(rcfg.vocab_size), device=torch.device("cpu"), ctx=ctx,
        config=rcfg, num_pages=num_pages, cache_manager=mods.cache.CacheManager(torch.device("cpu"), num_pages),
    )
