"""The drop-in boundary on the GPU: reference configuration names and plugin
slots reach the sm_100a kernels unchanged.

* AttnRes backend slot: ``LLM(..., attnres_backend=name)`` with each of the
  reference's names (aios/models/config.py:27,34-40; aios/llm/llm.py:38-40) runs
  the one fused sm_100a mixer, so a keystroke gives the same candidates, bit for
  bit, whichever name a caller passes.
"""

from __future__ import annotations

import dataclasses

import pytest
import torch

from aios_b200 import ImeCompletionEngine, ImeGenerationConfig, LLM
from aios_b200.models import shapes

pytestmark = pytest.mark.gpu

S21_L4 = dataclasses.replace(shapes.S21, num_layers=4, attnres_num_blocks=2)


def _keystroke(backend: str | None) -> list[tuple[str, float]]:
    kwargs = {} if backend is None else {"attnres_backend": backend}
    llm = LLM(config=S21_L4, seed=0, page_size=16, num_pages=64, **kwargs)
    assert llm.config.attnres_backend == (backend or S21_L4.attnres_backend)
    engine = ImeCompletionEngine(llm)
    g = torch.Generator().manual_seed(5)
    text = llm.tokenizer.text_for(torch.randint(10, S21_L4.vocab_size, (12,), generator=g).tolist())
    result = engine.complete(text, ImeGenerationConfig(seed=4, max_new_tokens=8))
    out = [(c.text, c.average_logprob) for c in result.raw_candidates]
    del engine, llm
    torch.cuda.empty_cache()
    return out


def test_reference_attnres_backend_names_run_the_b200_mixer() -> None:
    want = _keystroke("b200")
    assert len(want) >= 8
    for name in (None, "triton", "reference", "eager", "compiled"):
        assert _keystroke(name) == want, name


def test_unknown_attnres_backend_name_is_rejected() -> None:
    with pytest.raises(ValueError, match="attnres_backend must be"):
        LLM(config=S21_L4, seed=0, page_size=16, num_pages=64, attnres_backend="flash")
