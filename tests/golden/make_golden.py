"""Generates the golden fixtures of tests/golden/ by running the UNMODIFIED
reference implementation (7155/aios, Python) on the CPU.

The reference's GPU-only pieces are replaced by the shims of
oracle/reference_run.py (the same ones bench.py's reference arm uses):
  1. FlashInfer rmsnorm / fused_add_rmsnorm / silu_and_mul -> torch expressions of
     FlashInfer's arithmetic (fp32 math, one rounding to the storage dtype);
  2. the attention backend -> a CPU backend that stores K/V in a
     [2, L, pages, 1, Hkv, d] buffer and calls the reference's own
     _sdpa_prefill_attention for prefill and decode;
  3. torch.cuda.Event -> a host-clock event;
  4. the tokenizer -> aios_b200's SyntheticTokenizer (ids <-> CJK characters).
Weights are the seeded synthetic weights of the benchmark protocol.

Usage (only where the reference checkout exists; the fixtures are committed):
    AIOS_REFERENCE=<reference checkout>/python python tests/golden/make_golden.py
"""

from __future__ import annotations

import dataclasses
import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("AIOS_REFERENCE"):
    raise SystemExit("set AIOS_REFERENCE to the reference checkout's python/ directory (the one holding aios/)")
REF = Path(os.environ["AIOS_REFERENCE"])
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

from oracle import reference_run  # noqa: E402  (the shims: FlashInfer norms, CPU attention + KV, host events)

_mods = reference_run.install(REF)
ref_core = _mods.core
ref_sample = _mods.sample
ImeCompletionEngine = _mods.ime.ImeCompletionEngine
ImeGenerationConfig = _mods.ime.ImeGenerationConfig
BlockAttnResMixer = _mods.minimind.BlockAttnResMixer
_sdpa_prefill_attention = _mods.attn_fi._sdpa_prefill_attention

from aios_b200.models import shapes  # noqa: E402
from aios_b200.models.weight import synthetic_state_dict  # noqa: E402
from aios_b200.tokenizer import SyntheticTokenizer  # noqa: E402


def build_llm(cfg, dtype, num_pages: int):
    fields = {f.name: getattr(cfg, f.name) for f in dataclasses.fields(cfg) if f.name != "attnres_backend"}
    with torch.device("meta"):
        model = _mods.minimind.MiniMindIMEForCausalLM(_mods.config.ModelConfig(**fields, attnres_backend="eager"))
    return reference_run.build_llm(_mods, fields, num_pages, dtype=dtype, state=synthetic_state_dict(model, seed=0),
                                   tokenizer=SyntheticTokenizer(cfg.vocab_size))


class Recorder:
    """Hooks that record what the reference engine did, step by step."""

    def __init__(self):
        self.events = []

    def install(self):
        rec = self
        orig_sample = ref_sample.Sampler.sample_with_logprobs
        orig_decode = ImeCompletionEngine._decode_step
        orig_branch = ImeCompletionEngine._generate_branch_batch

        def sample(self, logits, **kw):
            tok, lp = orig_sample(self, logits, **kw)
            rec.events.append(("sample", tok.squeeze(-1).tolist(), lp.squeeze(-1).tolist()))
            return tok, lp

        def decode(self, token_ids, page_table, *, cached_len, row_indices):
            logits, pages = orig_decode(self, token_ids, page_table, cached_len=cached_len, row_indices=row_indices)
            rec.events.append(("decode", token_ids.tolist(), cached_len, row_indices.tolist(), pages.tolist()))
            return logits, pages

        def branch(self, **kw):
            rec.events.append(("round", dict(
                row_offset=kw["row_offset"], attempts=kw["attempts"], seed=kw["seed"],
                temperature=kw["temperature"], top_k=kw["top_k"], top_p=kw["top_p"],
                forbidden=[list(s) for s in kw["forbidden_sequences"]],
            )))
            return orig_branch(self, **kw)

        ref_sample.Sampler.sample_with_logprobs = sample
        ImeCompletionEngine._decode_step = decode
        ImeCompletionEngine._generate_branch_batch = branch
        import aios.ime as ref_ime

        ref_ime.Sampler = ref_sample.Sampler

    def take(self):
        out, self.events = self.events, []
        return out


# ---------------------------------------------------------------------------
# fixtures
# ---------------------------------------------------------------------------
SAMPLER_CASES = [
    dict(temperature=0.8, top_k=50, top_p=0.9),
    dict(temperature=0.75, top_k=96, top_p=0.95),
    dict(temperature=0.35, top_k=50, top_p=1.0),
    dict(temperature=0.9, top_k=-1, top_p=0.9),
    dict(temperature=1.0, top_k=-1, top_p=1.0),
    dict(temperature=0.5, top_k=1, top_p=1.0),
    dict(temperature=0.0, top_k=-1, top_p=1.0),
]


def gen_sampler() -> dict:
    g = torch.Generator().manual_seed(1234)
    logits = torch.randn(16, 2048, generator=g) * 3.0  # fp32: no ties, tie order irrelevant
    seeds = [20260814 + i for i in range(16)]
    uniforms = ref_sample.stateless_uniforms(seeds, 5, torch.device("cpu"))
    ban_rows = torch.randint(0, 2048, (16, 3), generator=g)
    out = {"logits": logits, "seeds": seeds, "uniforms": uniforms, "ban_rows": ban_rows, "cases": []}
    for case in SAMPLER_CASES:
        sp = ref_core.SamplingParams(**case)
        s = ref_sample.Sampler(sp)
        tok, lp = s.sample_with_logprobs(logits, uniforms=uniforms[:, 2], forbidden_token_ids=(3, 7, 11),
                                         forbidden_token_ids_by_row=ban_rows)
        out["cases"].append(dict(params=case, tokens=tok.squeeze(-1), logprobs=lp.squeeze(-1)))
    big = [2**63 - 5, 2**64 - 1, 0, 17, 20260814 + 3 * 100003]
    out["uniform_seeds"] = big
    out["uniform_values"] = ref_sample.stateless_uniforms(big, 24, torch.device("cpu"))
    return out


def gen_mixer() -> dict:
    """the 65-mixer dependency chain of
    benchmark/profile_attnres.py (banks of depth 1..9 + one partial), [8, 768],
    N(0,1) sources, query N(0, 0.02), norm weight 1, seed 0, fp32, eager backend."""
    g = torch.Generator().manual_seed(0)
    banks = [torch.randn(depth, 8, 768, generator=g) for depth in range(1, 10)]
    partial = torch.randn(8, 768, generator=g)
    queries = [torch.randn(768, generator=g) * 0.02 for _ in range(65)]
    outputs = []
    idx = 0

    def mix(bank, part):
        nonlocal idx
        m = BlockAttnResMixer(768, 1e-6, "eager")
        m.query = queries[idx].clone()
        m.key_norm.weight = torch.ones(768)
        idx += 1
        return m.forward(bank, part)

    for block in range(8):
        for layer in range(4):
            outputs.append(mix(banks[block], None if layer == 0 else partial))
            outputs.append(mix(banks[block], partial))
    outputs.append(mix(banks[8], None))
    stats = torch.stack([torch.stack([o.sum(), o.square().sum(), o.abs().max()]) for o in outputs])
    keep = [0, 1, 7, 31, 64]
    return {"keep": keep, "outputs": torch.stack([outputs[i] for i in keep]), "stats": stats}


def gen_attention() -> dict:
    g = torch.Generator().manual_seed(17)
    cases = []
    for cached in (0, 2, 9):
        n = 5
        q = torch.randn(n, 8, 96, generator=g)
        k = torch.randn(cached + n, 2, 96, generator=g)
        v = torch.randn(cached + n, 2, 96, generator=g)
        out = _sdpa_prefill_attention(q, k, v, cached_len=cached, sm_scale=96**-0.5)
        cases.append(dict(cached=cached, q=q, k=k, v=v, out=out))
    return {"cases": cases}


def _keystroke(engine, llm, rec, prefix_ids, cfg):
    text = llm.tokenizer.text_for(prefix_ids[1:])
    result = engine.complete(text, cfg)
    events = rec.take()
    return dict(
        prefix_ids=prefix_ids,
        events=events,
        page_table=llm.ctx.page_table.clone(),
        free_after=llm.cache_manager._free_slots.clone(),
        prefix_logits=engine._prefix_logits.float().clone(),
        result=dict(
            candidates=[c.text for c in result.candidates],
            raw=[(c.text, c.token_count, c.average_logprob, c.base_score, c.stop_reason, c.invalid_reasons)
                 for c in result.raw_candidates],
            sampling_attempts=result.sampling_attempts, generated_tokens=result.generated_tokens,
            active_model_tokens=result.active_model_tokens, unique_kv_pages=result.unique_kv_pages,
            reused_prefix_tokens=result.reused_prefix_tokens, refill_rounds=result.refill_rounds,
            refill_stop_reason=result.refill_stop_reason,
        ),
    )


def gen_model(name: str, cfg, dtype, rec: Recorder) -> dict:
    """A reduced-depth model of a benchmark shape: one keystroke stream through
    the reference engine (prefill, LCP extension, identical repeat, backspace),
    plus a refill run and a greedy run."""
    llm = build_llm(cfg, dtype, num_pages=1024)
    engine = ImeCompletionEngine(llm)
    rec.take()  # drop events of earlier fixtures
    g = torch.Generator().manual_seed(0)
    base = [1] + torch.randint(10, cfg.vocab_size, (14,), generator=g).tolist()
    sampled = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                                  max_new_tokens=6, temperature=0.8, seed=0)
    keystrokes = []
    for ids in (base[:11], base[:13], base[:13], base[:12], base):
        keystrokes.append(_keystroke(engine, llm, rec, ids, sampled))
    refill = ImeGenerationConfig(sampling_attempts=4, max_sampling_attempts=12, refill_batch_size=4,
                                 min_refill_batch_size=2, max_new_tokens=5, temperature=0.8, seed=5)
    keystrokes.append(_keystroke(engine, llm, rec, base[:9], refill))
    greedy = ImeGenerationConfig(sampling_attempts=4, max_sampling_attempts=4, refill_batch_size=4,
                                 max_new_tokens=6, temperature=1.0, top_k=1, top_p=1.0, min_new_tokens=0, seed=2)
    keystrokes.append(_keystroke(engine, llm, rec, base[:10], greedy))
    return {"name": name, "config": {f.name: getattr(cfg, f.name) for f in dataclasses.fields(cfg)},
            "dtype": str(dtype), "num_pages": 1024,
            "configs": {"sampled": dataclasses.asdict(sampled), "refill": dataclasses.asdict(refill),
                        "greedy": dataclasses.asdict(greedy)},
            "keystrokes": keystrokes}


def reduced(cfg, layers: int, **extra):
    return dataclasses.replace(cfg, num_layers=layers, **extra)


def main(out_dir: Path = HERE) -> None:
    torch.manual_seed(0)
    rec = Recorder()
    rec.install()
    torch.save(gen_sampler(), out_dir / "sampler.pt")
    torch.save(gen_mixer(), out_dir / "mixer.pt")
    torch.save(gen_attention(), out_dir / "attention.pt")
    models = {
        "s10_l2_fp32": (reduced(shapes.S10, 2), torch.float32),
        "s10_l2_bf16": (reduced(shapes.S10, 2), torch.bfloat16),
        "s06_l2_fp32": (reduced(shapes.S06, 2), torch.float32),
        "s21_l4_fp32": (reduced(shapes.S21, 4, attnres_num_blocks=2), torch.float32),
    }
    for key, (cfg, dtype) in models.items():
        torch.save(gen_model(key, cfg, dtype, rec), out_dir / f"model_{key}.pt")
        print("wrote", key)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
