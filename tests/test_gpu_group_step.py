"""One CandidateGroup step (aiosb_group_step) on given logits, every sampling
branch, against the oracle sampler (aios/engine/sample.py:54-163 with the
minimum-length bans of aios/ime.py:1008-1012).

One CTA samples a row by default; with AIOSB_GROUP_SPLIT a cluster of CTAs
splits each row on the top-k path (k <= 512) and falls back to one CTA for
greedy, top-p without top-k, larger k, rows whose candidate set overflows (ties)
and values that the temperature could overflow; each branch has a case here, run
in process (one CTA) and in child processes with 2, 4 and 8 CTAs per row. Tokens are bit-exact (a mismatch only at
a CDF-boundary rounding tie), log-probabilities within 2e-5."""

from __future__ import annotations

import ctypes

import pytest
import torch

from aios_b200 import _lib
from oracle import sampler as osamp

pytestmark = pytest.mark.gpu

ROWS, STEPS, WIDTH = 8, 4, 64
MINLEN = [2, 7, 100, 5000]  # forbidden at step 0 (min_new_tokens 1); 2 is EOS


def _group(dev, vocab: int, *, temperature: float, top_k: int, top_p: float, greedy: bool) -> dict:
    i32 = dict(dtype=torch.int32, device=dev)
    b = dict(
        state=torch.zeros(ctypes.sizeof(_lib.GroupState), dtype=torch.uint8, device=dev),
        logits=torch.zeros((ROWS, vocab), dtype=torch.bfloat16, device=dev),
        uniforms=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        output_ids=torch.zeros((ROWS, STEPS), **i32),
        token_logprobs=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        logprob_sums=torch.zeros(ROWS, dtype=torch.float32, device=dev),
        terminal_ids=torch.tensor([-1], **i32),
        minlen_ids=torch.tensor(MINLEN, **i32),
        page_table=torch.zeros((ROWS, WIDTH), **i32),
        ring=torch.arange(64, **i32),
        status=torch.zeros(1, **i32),
    )
    for name in ("counts", "stop_codes", "active", "finished", "tokens", "positions", "seq_lens", "out_loc",
                 "row_page", "row_table"):
        b[name] = torch.zeros(ROWS, **i32)
    st = _lib.GroupState(step=0, max_steps=STEPS, min_new_tokens=1, prefix_len=5, rows=ROWS, vocab=vocab, eos_id=2,
                         pad_id=0, greedy=int(greedy), top_k=top_k, temperature=temperature, top_p=top_p,
                         page_size=1, n_terminal=0, n_minlen=len(MINLEN), head=0, tail=64, capacity=64,
                         table_stride=WIDTH)
    b["state"].copy_(torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8))
    fields = {name for name, _ in _lib.GroupPtrs._fields_}
    b["ptrs"] = _lib.GroupPtrs(**{k: v.data_ptr() for k, v in b.items() if k in fields})
    return b


def _logits(mode: str, vocab: int, g: torch.Generator) -> torch.Tensor:
    if mode == "const":
        return torch.zeros(ROWS, vocab).to(torch.bfloat16)
    if mode == "coarse":
        return torch.randint(-3, 4, (ROWS, vocab), generator=g).float().to(torch.bfloat16)
    x = torch.randn(ROWS, vocab, generator=g) * 2.0
    if mode == "huge":  # finite after scaling, above the raw-key bound
        idx = torch.randint(0, vocab, (ROWS, 3), generator=g)
        x = x.scatter(1, idx, torch.tensor([1e38, -1e38, 6e37]).expand(ROWS, 3))
    return x.to(torch.bfloat16)


CASES = [
    # name, vocab, temperature, top_k, top_p, greedy, logits
    ("split_k50", 16384, 0.8, 50, 0.9, False, "randn"),
    ("split_k1_sampled", 16384, 0.8, 1, 0.9, False, "randn"),
    ("split_k512", 16384, 1.0, 512, 0.95, False, "randn"),
    ("split_s06_vocab", 6400, 0.8, 50, 0.9, False, "randn"),
    ("split_ragged_vocab", 6401, 0.7, 96, 0.9, False, "randn"),
    ("split_small_vocab", 600, 0.8, 200, 0.9, False, "randn"),
    ("split_few_distinct", 16384, 0.8, 50, 1.0, False, "coarse"),
    ("overflow_ties", 16384, 0.8, 50, 0.9, False, "const"),
    ("hazard_huge", 16384, 0.5, 50, 0.9, False, "huge"),
    ("one_cta_k600", 16384, 0.8, 600, 0.9, False, "randn"),
    ("one_cta_topp_only", 16384, 0.8, 0, 0.9, False, "randn"),
    ("one_cta_greedy", 16384, 1.0, 1, 1.0, True, "randn"),
]


@pytest.mark.parametrize("name,vocab,temperature,top_k,top_p,greedy,mode", CASES, ids=[c[0] for c in CASES])
def test_group_step_matches_oracle_sampler(cuda_device, name, vocab, temperature, top_k, top_p, greedy,
                                           mode) -> None:
    g = torch.Generator().manual_seed(len(name) * 31 + vocab)
    grp = _group(cuda_device, vocab, temperature=temperature, top_k=top_k, top_p=top_p, greedy=greedy)
    logits = _logits(mode, vocab, g)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    _lib.call("aiosb_group_begin", ctypes.byref(grp["ptrs"]), grp["logits"][0].clone().data_ptr(), 1234 + vocab,
              ROWS, ROWS, stream)
    grp["logits"].copy_(logits.to(cuda_device))  # per-row logits over the broadcast prefix row
    top_k_max = vocab if top_k == 0 else top_k
    _lib.call("aiosb_group_step", ctypes.byref(grp["ptrs"]), ROWS, vocab, top_k_max, stream)
    torch.cuda.synchronize(cuda_device)
    assert int(grp["status"][0]) == 0
    u = grp["uniforms"][:, 0].cpu()
    minlen = [t for t in MINLEN if t < vocab]  # ids outside the vocabulary are ignored (aios/ime.py:1008-1012)
    exp_tok, exp_lp = osamp.sample_with_logprobs(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                                 uniforms=u, forbidden_token_ids=minlen)
    tok = grp["tokens"].cpu().long()
    mism = tok != exp_tok.squeeze(-1)
    if bool(mism.any()):
        bans = dict(forbidden_token_ids=minlen)
        margins = osamp.sample_margin(logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u, **bans)
        band = osamp.cdf_rounding_band(logits, temperature=temperature, top_k=top_k, top_p=top_p, **bans)
        bad = (margins >= band + 1e-6) & mism.numpy()
        assert not bad.any(), f"{name}: token mismatch rows {bad.nonzero()[0].tolist()}"
    # EOS is forbidden at step 0, so every row emitted its token
    assert grp["output_ids"][:, 0].cpu().long().tolist() == tok.tolist()
    assert grp["counts"].cpu().tolist() == [1] * ROWS
    lp = grp["token_logprobs"][:, 0].cpu()
    ref = torch.log_softmax(logits.float(), dim=-1).gather(1, tok[:, None])[:, 0]
    torch.testing.assert_close(lp, ref, rtol=0, atol=2e-5)
    if not mism.any():
        torch.testing.assert_close(lp, exp_lp.squeeze(-1), rtol=0, atol=2e-5)
    # the step epilogue ran once: one FIFO slot per row, in row order
    assert grp["out_loc"].cpu().tolist() == list(range(ROWS))


@pytest.mark.parametrize("split", [2, 4, 8])
def test_group_step_other_cluster_sizes(split: int) -> None:
    """The same cases with rows split over 2, 4 and 8 CTAs (the library reads the
    split once, at load: a child process per size)."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    env = dict(os.environ, AIOSB_GROUP_SPLIT=str(split))
    proc = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
                           str(Path(__file__).resolve()), "-k", "matches_oracle"],
                          cwd=repo, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]
