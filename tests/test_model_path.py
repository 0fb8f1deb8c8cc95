"""A model directory end to end: ``LLM(model_path)`` reads config.json, the
safetensors shards (Hugging Face layout: separate q/k/v and gate/up) and a
tokenizer.json through ``transformers.AutoTokenizer``, as the reference does
(aios/llm/llm.py:27-75, aios/models/weight.py:48-70; its GPU tests drive a real
checkpoint the same way, tests/test_ime_gpu.py:28-87). No MiniMind-IME
checkpoint exists offline, so the directory is written here: the seeded
synthetic weights, and a word-level tokenizer (one token per character, <pad> 0,
<s> 1, </s> 2) whose ids equal the synthetic tokenizer's.

* CPU: the written tokenizer loads through AutoTokenizer and encodes / decodes
  exactly as the synthetic tokenizer.
* GPU: a keystroke through the model directory gives the same candidates and
  scores as the same weights built in memory.
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import pytest
import torch

from aios_b200.models import shapes
from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM
from aios_b200.models.weight import synthetic_state_dict
from aios_b200.tokenizer import SyntheticTokenizer
from tests.test_checkpoint import _hf_config, _hf_tensors

CFG = dataclasses.replace(shapes.S10, num_layers=2)


def write_tokenizer(path: Path, vocab_size: int) -> None:
    """tokenizer.json + tokenizer_config.json: a word-level model over single
    characters with the synthetic tokenizer's ids."""
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers

    ref = SyntheticTokenizer(vocab_size)
    vocab = {"<pad>": 0, "<s>": 1, "</s>": 2}
    vocab.update({ref.id_to_char(i): i for i in range(3, vocab_size)})
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = pre_tokenizers.Split(Regex("."), behavior="isolated")
    tok.decoder = decoders.Fuse()
    tok.add_special_tokens(["<pad>", "<s>", "</s>"])
    tok.save(str(path / "tokenizer.json"))
    (path / "tokenizer_config.json").write_text(json.dumps({
        "tokenizer_class": "PreTrainedTokenizerFast", "bos_token": "<s>", "eos_token": "</s>",
        "pad_token": "<pad>", "unk_token": "<pad>", "clean_up_tokenization_spaces": False,
    }))


def write_model_dir(path: Path, cfg=CFG, seed: int = 0) -> Path:
    from safetensors.torch import save_file

    path.mkdir(parents=True, exist_ok=True)
    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    tensors = _hf_tensors(cfg, synthetic_state_dict(meta, seed=seed))
    names = sorted(tensors)
    save_file({n: tensors[n] for n in names[::2]}, str(path / "model-00001-of-00002.safetensors"))
    save_file({n: tensors[n] for n in names[1::2]}, str(path / "model-00002-of-00002.safetensors"))
    conf = _hf_config(cfg)
    conf["model_type"] = "minimind_ime_v3"
    (path / "config.json").write_text(json.dumps(conf))
    write_tokenizer(path, cfg.vocab_size)
    return path


def test_written_tokenizer_matches_the_synthetic_one(tmp_path) -> None:
    from transformers import AutoTokenizer

    write_tokenizer(tmp_path, CFG.vocab_size)
    auto = AutoTokenizer.from_pretrained(str(tmp_path))
    ref = SyntheticTokenizer(CFG.vocab_size)
    text = ref.text_for([10, 523, 16383, 4, 77, 3]) + "今天"
    assert auto.encode(text, add_special_tokens=False) == ref.encode(text)
    ids = ref.encode(text)
    assert auto.decode(ids, skip_special_tokens=True) == ref.decode(ids)
    assert auto.decode([1, *ids, 2, 0], skip_special_tokens=True) == ref.decode(ids)
    assert (auto.bos_token_id, auto.eos_token_id, auto.pad_token_id) == (1, 2, 0)


@pytest.mark.gpu
def test_keystroke_through_a_model_directory(tmp_path) -> None:
    from aios_b200 import ImeCompletionEngine, ImeGenerationConfig, LLM

    model_dir = write_model_dir(tmp_path / "minimind-ime-s10-l2")
    cfg = ImeGenerationConfig(seed=3, max_new_tokens=8)
    text = SyntheticTokenizer(CFG.vocab_size).text_for([11, 2000, 5000, 9000, 123, 456])

    llm = LLM(str(model_dir), page_size=16, num_pages=64)
    assert type(llm.tokenizer).__name__ != "SyntheticTokenizer"
    assert llm.config.num_layers == 2 and llm.config.vocab_size == CFG.vocab_size
    got = ImeCompletionEngine(llm).complete(text, cfg)
    got_raw = [(c.text, c.token_count, c.average_logprob) for c in got.raw_candidates]
    del llm
    torch.cuda.empty_cache()

    mem = LLM(config=CFG, seed=0, page_size=16, num_pages=64)
    want = ImeCompletionEngine(mem).complete(text, cfg)
    assert got.prefix_tokens == want.prefix_tokens == 7
    assert got_raw == [(c.text, c.token_count, c.average_logprob) for c in want.raw_candidates]
    assert [c.text for c in got.candidates] == [c.text for c in want.candidates]
