"""One small CandidateGroup keystroke on cuda:0, checked against the CPU oracle.

Runs a 2-layer model of the 0.1B IME shape through ``ImeCompletionEngine.complete``
(16-token pages) and replays every sampling round on the oracle with the GPU's
own step logits: tokens bit for bit, log-probabilities within the bf16 bound,
page-table entries and the free-slot FIFO bit for bit. Raises on any mismatch.
"""

from __future__ import annotations

import dataclasses
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def run_smoke() -> dict:
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("smoke() needs a CUDA device")
    torch.cuda.set_device(0)
    from aios_b200 import ImeGenerationConfig, _lib
    from aios_b200.models import shapes
    from tests.test_gpu_parity import _check_keystroke, _models

    cfg = dataclasses.replace(shapes.S10, num_layers=2)
    llm, engine, oeng = _models(cfg, page_size=16, num_pages=128)
    g = torch.Generator().manual_seed(0)
    ids = [1] + torch.randint(10, cfg.vocab_size, (11,), generator=g).tolist()
    gen = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                              max_new_tokens=6, temperature=0.8, seed=0)
    stats: dict = {}
    before = _lib.launches
    _check_keystroke(llm, engine, oeng, ids, gen, stats)
    torch.cuda.synchronize()
    stats["library_launches"] = _lib.launches - before
    if stats.get("tokens", 0) == 0 or stats["library_launches"] == 0:
        raise RuntimeError(f"smoke keystroke produced no work: {stats}")
    print("smoke ok", stats)
    return stats


if __name__ == "__main__":
    run_smoke()
