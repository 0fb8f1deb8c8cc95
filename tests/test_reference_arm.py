"""The reference arm of bench.py: the unmodified reference engine on the CPU.

* The runner (oracle/reference_run.py: the installed reference package plus four
  CPU shims) reproduces the committed golden keystrokes, which the fixture
  generator made from the reference checkout: candidates, raw candidate scores,
  the page table and the free-slot FIFO, bit for bit.
* ``bench.py --impl reference`` prints a "reference"-kind line with the GPU arm's
  config and never imports the product package or maps its library.

Both need the reference installed under baseline/_ref (``pip install --target``);
without it they are skipped.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
INSTALL = REPO / "baseline" / "_ref"
GOLDEN = REPO / "tests" / "golden"

pytestmark = pytest.mark.skipif(not (INSTALL / "aios" / "ime.py").exists(),
                                reason="reference not installed under baseline/_ref")


@pytest.fixture
def reference(monkeypatch):
    """The shimmed reference modules; the process-global shims are undone after."""
    from oracle import reference_run

    monkeypatch.setattr(torch.cuda, "Event", torch.cuda.Event)
    try:
        import flashinfer

        for name in ("rmsnorm", "fused_add_rmsnorm", "silu_and_mul"):
            monkeypatch.setattr(flashinfer, name, getattr(flashinfer, name))
    except ImportError:
        pass
    monkeypatch.syspath_prepend(str(INSTALL))
    return reference_run, reference_run.install(INSTALL)


@pytest.mark.parametrize("fixture", ["model_s10_l2_fp32.pt", "model_s21_l4_fp32.pt"])
def test_reference_runner_reproduces_golden_keystrokes(reference, fixture) -> None:
    rr, mods = reference
    gold = torch.load(GOLDEN / fixture, weights_only=False)
    fields = {k: v for k, v in gold["config"].items() if k != "attnres_backend"}
    llm = rr.build_llm(mods, fields, num_pages=gold["num_pages"], dtype=torch.float32)
    engine = mods.ime.ImeCompletionEngine(llm)
    cfgs = {name: mods.ime.ImeGenerationConfig(**c) for name, c in gold["configs"].items()}
    order = ["sampled"] * 5 + ["refill", "greedy"]
    for ks, cfg_name in zip(gold["keystrokes"], order):
        result = engine.complete(llm.tokenizer.text_for(ks["prefix_ids"][1:]), cfgs[cfg_name])
        want = ks["result"]
        assert [c.text for c in result.candidates] == want["candidates"]
        raw = [(c.text, c.token_count, c.average_logprob, c.base_score, c.stop_reason, c.invalid_reasons)
               for c in result.raw_candidates]
        assert raw == want["raw"]
        assert result.sampling_attempts == want["sampling_attempts"]
        assert result.reused_prefix_tokens == want["reused_prefix_tokens"]
        assert torch.equal(llm.ctx.page_table, ks["page_table"])
        assert torch.equal(llm.cache_manager._free_slots, ks["free_after"])


def test_bench_reference_arm_runs_the_reference_without_product_code() -> None:
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('PRODUCT', 'libaios_b200' in maps or any(m.split('.')[0] == 'aios_b200' for m in sys.modules))\n"
    )
    proc = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = proc.stdout.strip().splitlines()
    line = json.loads(next(x for x in lines if x.startswith("{")))
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "reference"
    assert line["config"]["model"] == "MiniMind-IME 0.1B shape (S10)" and line["unit"] == "keystrokes/s"
    assert lines[-1] == "PRODUCT False"
