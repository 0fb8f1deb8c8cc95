"""The persistent decode step (aiosb_decode_step) on the GPU.

* Against the per-kernel forward: the same greedy keystroke through both decode
  paths, every step's logits recorded. The two paths sum some products in a
  different order (the down projection splits its 2048-long K differently), so
  bf16 outputs can round apart and the difference grows over steps; the bar is
  the drift measured between two faithful CPU restatements that differ only in
  summation order (fp32 vs fp64 accumulation): two bf16 ulps of the row's
  largest logit over the whole vocabulary. A wrong tile, head or layer would
  show as differences orders of magnitude larger. Greedy tokens agree except
  where the top-2 logit gap is a bf16 near-tie.
* Bounded waits: a launch whose phases expect a flag no producer writes (the test
  hook test_flag_skew), with a 2 ms limit, reports AIOSB_DEV_WAIT_TIMEOUT through
  the status word and returns; the abort and launch-counter words are left at
  zero, and the next ordinary launch works.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from aios_b200 import ImeCompletionEngine, ImeGenerationConfig, LLM, _lib
from aios_b200.kernel import ops
from aios_b200.models import shapes

pytestmark = pytest.mark.gpu


def _greedy_steps(engine, text: str, cfg) -> list[torch.Tensor]:
    rt = engine._runtime
    rt.record, rt.record_logits = True, True
    rt.rounds.clear()
    engine.reset_prefix_cache()
    engine.complete(text, cfg)
    (params, res), = rt.rounds
    return params["step_logits"], res


@pytest.mark.parametrize("shape", ["S10", "S06"])
def test_persistent_step_matches_per_kernel_forward(shape) -> None:
    cfg = getattr(shapes, shape)
    llm = LLM(config=cfg, seed=0, page_size=16, num_pages=256)
    engine = ImeCompletionEngine(llm)
    rt = engine._runtime
    assert rt.use_persistent_step(), "the persistent step should serve this shape"
    g = torch.Generator().manual_seed(9)
    text = llm.tokenizer.text_for(torch.randint(10, cfg.vocab_size, (12,), generator=g).tolist())
    greedy = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                                 max_new_tokens=12, temperature=1.0, top_k=1, top_p=1.0, min_new_tokens=0, seed=1)
    persistent, res_p = _greedy_steps(engine, text, greedy)
    launches = rt._graph_launches[(8, False, 128)]
    rt.use_persistent_step(False)  # the per-kernel forward, same weights and buffers
    per_kernel, res_k = _greedy_steps(engine, text, greedy)
    assert launches == 2, "one group step + one persistent forward per decode step"
    assert rt._graph_launches[(8, False, 128)] > 2 * cfg.num_layers
    steps = min(len(persistent), len(per_kernel))
    assert steps >= 2
    worst = 0.0
    for s in range(steps):
        a, b = persistent[s], per_kernel[s]
        rows = min(a.shape[0], b.shape[0])
        diff = (torch.log_softmax(a[:rows], -1) - torch.log_softmax(b[:rows], -1)).abs().max().item()
        worst = max(worst, diff)
        ulp = 2.0 ** (math.floor(math.log2(float(b[:rows].abs().max()))) - 7)
        assert diff <= 2 * ulp + 1e-3, (s, diff, ulp)
    flips = 0
    for r in range(8):
        n = min(res_p.counts[r], res_k.counts[r])
        for s in range(n):
            if res_p.output_ids[r, s] != res_k.output_ids[r, s]:
                top2 = per_kernel[s][r].topk(2).values
                assert float(top2[0] - top2[1]) < 2e-2, (r, s)
                flips += 1
                break
    print(shape, "persistent vs per-kernel: max log-softmax diff", worst, "greedy divergences", flips)


def test_decode_step_wait_runs_out_and_reports() -> None:
    llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=64)
    engine = ImeCompletionEngine(llm)
    rt = engine._runtime
    assert rt.use_persistent_step()
    plan = rt._step_plan
    dev = llm.device
    status = ops.status_word(dev)
    torch.cuda.synchronize(dev)
    status.zero_()
    args = _lib.DecodeStepArgs.from_buffer_copy(plan["args"])
    args.rows = 8
    args.wait_limit_ns = 2_000_000  # 2 ms
    args.test_flag_skew = 1  # every wait expects a flag that no producer writes
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.call("aiosb_decode_step", ctypes.byref(args), stream)
    torch.cuda.synchronize(dev)  # returns: every wait is bounded
    assert int(status.item()) == _lib.DEV_WAIT_TIMEOUT
    sync = plan["sync"].cpu().tolist()
    assert sync[0] == 0 and sync[1] == 0, "the last CTA clears the launch counter and the abort word"
    status.zero_()
    # the context is still usable: an ordinary launch completes and reports nothing
    ok = _lib.DecodeStepArgs.from_buffer_copy(plan["args"])
    ok.rows = 8
    _lib.call("aiosb_decode_step", ctypes.byref(ok), stream)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    after = plan["sync"].cpu().tolist()
    assert after[0] == 0 and after[1] == 0 and after[2] == sync[2] + 1, "one launch advances the flag epoch"
    assert torch.isfinite(rt.logits[:8].float()).all()
