"""One CandidateGroup step (aiosb_group_step) on given logits, every sampling
branch, against the oracle sampler (aios/engine/sample.py:54-163 with the
minimum-length bans of aios/ime.py:1008-1012).

One CTA samples a row by default; with AIOSB_GROUP_SPLIT a cluster of CTAs
splits each row on the top-k path (k <= 512) and falls back to one CTA for
greedy, top-p without top-k, larger k, rows whose candidate set overflows (ties)
and values that the temperature could overflow; each branch has a case here, run
in process (one CTA) and in child processes with 2, 4 and 8 CTAs per row. Tokens are bit-exact (a mismatch only at
a CDF-boundary rounding tie), log-probabilities within 2e-5.

Decode steps sample from the LM head's per-tile statistics; those cases compare
that path with the row scan (same tokens) and with the oracle, run the
after-forward form that reads the state before its wait (bit-identical), and
check that the step's embedding of the sampled tokens equals
aiosb_embedding_stat bit for bit."""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from aios_b200 import _lib
from oracle import sampler as osamp

pytestmark = pytest.mark.gpu

ROWS, STEPS, WIDTH = 8, 4, 64
MINLEN = [2, 7, 100, 5000]  # forbidden at step 0 (min_new_tokens 1); 2 is EOS


def _group(dev, vocab: int, *, temperature: float, top_k: int, top_p: float, greedy: bool, step: int = 0,
           min_new_tokens: int = 1) -> dict:
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
    st = _lib.GroupState(step=step, max_steps=STEPS, min_new_tokens=min_new_tokens, prefix_len=5, rows=ROWS, vocab=vocab, eos_id=2,
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
    if mode == "peaked":  # the largest values packed into four neighbouring tiles
        x[:, 512:576] += 8.0
    if mode == "banned_top":  # forbidden ids hold the largest values of their tiles
        x[:, [t for t in MINLEN if t < vocab]] += 12.0
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


def _tile_stats(logits: torch.Tensor) -> torch.Tensor:
    """[vocab / 16, rows, 4]: per 16-id tile of each row, the max, the sum of
    exp(v - max), the min and a NaN flag (what the LM head's epilogue writes)."""
    t = logits.float().view(logits.shape[0], -1, 16)
    mx = t.amax(-1)
    return torch.stack((mx, torch.exp(t - mx[..., None]).sum(-1), t.amin(-1), t.isnan().any(-1).float()),
                       -1).transpose(0, 1).contiguous()


TILE_CASES = [
    # name, vocab, temperature, top_k, top_p, logits, min_new_tokens (> 1: MINLEN forbidden at step 1)
    ("tiles_k50", 16384, 0.8, 50, 0.9, "randn", 2),
    ("tiles_k1_sampled", 16384, 0.8, 1, 0.9, "randn", 1),
    ("tiles_k512", 16384, 1.0, 512, 0.95, "randn", 2),
    ("tiles_s06_vocab", 6400, 0.8, 50, 0.9, "randn", 2),
    ("tiles_peaked", 16384, 0.8, 50, 0.9, "peaked", 1),
    ("tiles_banned_top", 16384, 0.8, 50, 0.9, "banned_top", 2),
    ("tiles_few_distinct", 16384, 0.8, 50, 1.0, "coarse", 2),  # more than 2048 candidates: the row scan
    ("tiles_ties", 16384, 0.8, 50, 0.9, "const", 2),  # every tile tied: the row scan
    ("tiles_hazard", 16384, 0.5, 50, 0.9, "huge", 2),  # values the temperature could overflow: the row scan
    ("tiles_more_than_tiles", 608, 0.8, 200, 0.9, "randn", 2),  # k + bans above the 38 tiles: the row scan
    ("tiles_ragged_vocab", 6401, 0.7, 96, 0.9, "randn", 2),  # vocab % 16 != 0: the row scan
]


def _run_step(dev, name, vocab, temperature, top_k, top_p, logits, min_new, tiles, after_forward=False):
    grp = _group(dev, vocab, temperature=temperature, top_k=top_k, top_p=top_p, greedy=False, step=1,
                 min_new_tokens=min_new)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.call("aiosb_group_begin", ctypes.byref(grp["ptrs"]), grp["logits"][0].clone().data_ptr(), 777 + vocab,
              ROWS, ROWS, stream)
    grp["logits"].copy_(logits.to(dev))
    if tiles is not None:
        grp["tiles"] = tiles.to(dev)
        grp["ptrs"].tile_stats = grp["tiles"].data_ptr()
    if after_forward:  # the state is read before the wait (the logits copy above is a plain kernel)
        grp["ptrs"].flags = _lib.GROUP_AFTER_FORWARD
    _lib.call("aiosb_group_step", ctypes.byref(grp["ptrs"]), ROWS, vocab, top_k, stream)
    torch.cuda.synchronize(dev)
    assert int(grp["status"][0]) == 0
    return grp


@pytest.mark.parametrize("name,vocab,temperature,top_k,top_p,mode,min_new", TILE_CASES,
                         ids=[c[0] for c in TILE_CASES])
def test_group_step_from_tile_statistics(cuda_device, name, vocab, temperature, top_k, top_p, mode,
                                         min_new) -> None:
    """A step after the first (logits written by the decode forward) with the LM
    head's tile statistics: the same tokens as the row scan and as the oracle,
    log-probabilities within 2e-5 of the exact log-softmax."""
    g = torch.Generator().manual_seed(len(name) * 17 + vocab)
    logits = _logits(mode, vocab, g)
    tiles = _tile_stats(logits) if vocab % 16 == 0 else torch.zeros(4)
    fast = _run_step(cuda_device, name, vocab, temperature, top_k, top_p, logits, min_new, tiles)
    scan = _run_step(cuda_device, name, vocab, temperature, top_k, top_p, logits, min_new, None)
    early = _run_step(cuda_device, name, vocab, temperature, top_k, top_p, logits, min_new, tiles, after_forward=True)
    # the after-forward form reads the same inputs earlier: the same results bit for bit
    assert torch.equal(early["tokens"], fast["tokens"])
    assert torch.equal(early["token_logprobs"], fast["token_logprobs"])
    tok = fast["tokens"].cpu().long()
    assert torch.equal(tok, scan["tokens"].cpu().long())
    assert fast["output_ids"][:, 1].cpu().long().tolist() == tok.tolist()
    u = fast["uniforms"][:, 1].cpu()
    bans = dict(forbidden_token_ids=[t for t in MINLEN if t < vocab] if min_new > 1 else [])
    exp_tok, _ = osamp.sample_with_logprobs(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                            uniforms=u, **bans)
    mism = tok != exp_tok.squeeze(-1)
    if bool(mism.any()):
        margins = osamp.sample_margin(logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u, **bans)
        band = osamp.cdf_rounding_band(logits, temperature=temperature, top_k=top_k, top_p=top_p, **bans)
        bad = (margins >= band + 1e-6) & mism.numpy()
        assert not bad.any(), f"{name}: token mismatch rows {bad.nonzero()[0].tolist()}"
    ref = torch.log_softmax(logits.float(), dim=-1).gather(1, tok[:, None])[:, 0]
    ok = torch.isfinite(ref)
    torch.testing.assert_close(fast["token_logprobs"][:, 1].cpu()[ok], ref[ok], rtol=0, atol=2e-5)


def test_group_step_reads_the_tile_statistics(cuda_device) -> None:
    """The top-k step takes its log-sum-exp from the tiles: doubling every tile's
    sum of exponentials lowers each log-probability by log 2, same tokens."""
    g = torch.Generator().manual_seed(3)
    logits = _logits("randn", 16384, g)
    tiles = _tile_stats(logits)
    doubled = tiles.clone()
    doubled[..., 1] *= 2.0
    a = _run_step(cuda_device, "a", 16384, 0.8, 50, 0.9, logits, 2, tiles)
    b = _run_step(cuda_device, "b", 16384, 0.8, 50, 0.9, logits, 2, doubled)
    assert torch.equal(a["tokens"], b["tokens"])
    lp_a, lp_b = a["token_logprobs"][:, 1].cpu(), b["token_logprobs"][:, 1].cpu()
    torch.testing.assert_close(lp_a - lp_b, torch.full((ROWS,), math.log(2.0)), rtol=0, atol=1e-5)


def test_group_step_embeds_the_sampled_tokens(cuda_device) -> None:
    """With the embedding fields set, each sampled row's next-forward input
    (embedding row, its fp32 copy and its sum of squares) equals
    aiosb_embedding_stat of the sampled token bit for bit; unsampled rows are
    left as they were."""
    from aios_b200.kernel import ops

    dev = cuda_device
    vocab, hidden = 16384, 768
    g = torch.Generator().manual_seed(11)
    grp = _group(dev, vocab, temperature=0.8, top_k=50, top_p=0.9, greedy=False)
    emb_w = torch.randn(vocab, hidden, generator=g).to(torch.bfloat16).to(dev)
    out = torch.full((ROWS, hidden), 7.0, dtype=torch.bfloat16, device=dev)
    sx = torch.full((ROWS, hidden), 7.0, device=dev)
    ss = torch.full((ROWS,), 7.0, device=dev)
    p = grp["ptrs"]
    p.embed_w, p.embed_out, p.embed_stat_x, p.embed_stat_ss, p.hidden = (
        emb_w.data_ptr(), out.data_ptr(), sx.data_ptr(), ss.data_ptr(), hidden)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.call("aiosb_group_begin", ctypes.byref(p), grp["logits"][0].clone().data_ptr(), 5, ROWS - 2, ROWS, stream)
    grp["logits"].copy_(_logits("randn", vocab, g).to(dev))
    _lib.call("aiosb_group_step", ctypes.byref(p), ROWS, vocab, 50, stream)
    torch.cuda.synchronize(dev)
    assert int(grp["status"][0]) == 0
    tok = grp["tokens"][: ROWS - 2].long()
    want_out, want_stats = ops.embedding_stat(tok, emb_w)
    torch.cuda.synchronize(dev)
    assert torch.equal(out[: ROWS - 2], want_out)
    assert torch.equal(sx[: ROWS - 2], want_stats.x)
    assert torch.equal(ss[: ROWS - 2], want_stats.ss[0])
    # the two rows the round did not start are not sampled and keep their contents
    assert bool((out[ROWS - 2 :].float() == 7.0).all()) and bool((ss[ROWS - 2 :] == 7.0).all())
    # a half-set embedding is refused on the host
    p.embed_out = 0
    with pytest.raises(ValueError, match="embed_w needs"):
        _lib.call("aiosb_group_step", ctypes.byref(p), ROWS, vocab, 50, stream)
