"""Oracle restatement of the reference sampler (TEST INFRASTRUCTURE ONLY).

Follows aios/engine/sample.py:12-163 step by step in CPU torch float32. The one
deliberate choice: ``tie_order``. torch.topk leaves the order of equal values
unspecified (its CPU partial sort is not stable), and that order decides which
token an inverse-CDF draw lands on inside a tie group. ``tie_order="index"``
orders equal logits by ascending token id (the B200 kernel's definition);
``tie_order="torch"`` calls torch.topk exactly like the reference (used to pin
this file against the reference's own outputs).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
import torch.nn.functional as F

MASK64 = (1 << 64) - 1


def splitmix64_uniform(seed: int, step: int) -> float:
    """aios/engine/sample.py:12-20."""
    value = (int(seed) + (int(step) + 1) * 0x9E3779B97F4A7C15) & MASK64
    value = ((value ^ (value >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    value = ((value ^ (value >> 27)) * 0x94D049BB133111EB) & MASK64
    value ^= value >> 31
    return (((value >> 11) & ((1 << 53) - 1)) + 0.5) / float(1 << 53)


def stateless_uniforms(seeds: Sequence[int], steps: int) -> torch.Tensor:
    """aios/engine/sample.py:23-45 (CPU tensor [rows, steps] float32)."""
    if steps < 1:
        raise ValueError("steps must be positive")
    return torch.tensor([[splitmix64_uniform(s, t) for t in range(steps)] for s in seeds], dtype=torch.float32)


def is_greedy(temperature: float, top_k: int, top_p: float) -> bool:
    """aios/core.py:22-24."""
    return (temperature <= 0.0 or top_k == 1) and top_p == 1.0


def _topk(scaled: torch.Tensor, k: int, tie_order: str) -> tuple[torch.Tensor, torch.Tensor]:
    if tie_order == "torch":
        return torch.topk(scaled, k)
    values, ids = torch.sort(scaled, dim=-1, descending=True, stable=True)
    return values[..., :k], ids[..., :k]


def sample_with_logprobs(
    logits: torch.Tensor,
    *,
    temperature: float,
    top_k: int,
    top_p: float,
    uniforms: torch.Tensor | None,
    forbidden_token_ids: Sequence[int] = (),
    forbidden_token_ids_by_row: torch.Tensor | None = None,
    tie_order: str = "index",
) -> tuple[torch.Tensor, torch.Tensor]:
    """aios/engine/sample.py:54-163 with explicit sampling parameters."""
    logits = logits.cpu()
    raw_log_probs = F.log_softmax(logits.float(), dim=-1)
    sampling_logits = logits.clone()
    if forbidden_token_ids:
        blocked = sorted({int(t) for t in forbidden_token_ids})
        sampling_logits[..., blocked] = -torch.inf
    if forbidden_token_ids_by_row is not None:
        row_ids = forbidden_token_ids_by_row.cpu().to(torch.long)
        if row_ids.numel():
            sampling_logits.scatter_(1, row_ids, -torch.inf)
    if is_greedy(temperature, top_k, top_p):
        token_ids = sampling_logits.argmax(dim=-1, keepdim=True)
        return token_ids, raw_log_probs.gather(-1, token_ids)
    scaled = sampling_logits.float() / temperature
    if top_k > 0:
        cand_logits, cand_ids = _topk(scaled, min(top_k, scaled.size(-1)), tie_order)
    elif top_p >= 1.0:
        cand_logits = scaled
        cand_ids = torch.arange(scaled.size(-1)).expand_as(scaled)
    else:
        cand_logits, cand_ids = _topk(scaled, scaled.size(-1), tie_order)
    probabilities = F.softmax(cand_logits, dim=-1)
    if top_p < 1.0:
        cumulative = probabilities.cumsum(dim=-1)
        remove = cumulative > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        cand_logits = cand_logits.masked_fill(remove, float("-inf"))
        probabilities = F.softmax(cand_logits, dim=-1)
    if uniforms is None:
        raise ValueError("the oracle samples with explicit uniforms only")
    u = uniforms.cpu().to(probabilities.dtype).unsqueeze(-1)
    sampled_index = (probabilities.cumsum(dim=-1) < u).sum(dim=-1, keepdim=True)
    sampled_index.clamp_max_(probabilities.size(-1) - 1)
    token_ids = cand_ids.gather(-1, sampled_index)
    return token_ids, raw_log_probs.gather(-1, token_ids)


def _sampling_cdfs(
    logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float,
    forbidden_token_ids: Sequence[int] = (), forbidden_token_ids_by_row: torch.Tensor | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """The candidate CDF of sample_with_logprobs in its own fp32 arithmetic, and
    the same CDF in fp64 over the fp32 path's candidates and top-p keep set."""
    sampling = logits.cpu().float().clone()
    if forbidden_token_ids:
        sampling[..., sorted({int(t) for t in forbidden_token_ids})] = -torch.inf
    if forbidden_token_ids_by_row is not None and forbidden_token_ids_by_row.numel():
        sampling.scatter_(1, forbidden_token_ids_by_row.cpu().to(torch.long), -torch.inf)
    scaled = sampling / temperature
    k = min(top_k, scaled.size(-1)) if top_k > 0 else scaled.size(-1)
    vals, _ = _topk(scaled, k, "index")
    probs = F.softmax(vals, dim=-1)
    if top_p < 1.0:
        remove = probs.cumsum(-1) > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        vals = vals.masked_fill(remove, float("-inf"))
        probs = F.softmax(vals, dim=-1)
    return probs.cumsum(-1).numpy(), torch.softmax(vals.double(), dim=-1).cumsum(-1).numpy()


def sample_margin(
    logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float, uniforms: torch.Tensor,
    forbidden_token_ids: Sequence[int] = (), forbidden_token_ids_by_row: torch.Tensor | None = None,
) -> np.ndarray:
    """Distance of each row's uniform from the nearest boundary of the fp32 CDF
    (diagnostics: a token mismatch with a tiny margin is a rounding tie, not a
    logic error)."""
    cdf, _ = _sampling_cdfs(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                            forbidden_token_ids=forbidden_token_ids,
                            forbidden_token_ids_by_row=forbidden_token_ids_by_row)
    return np.abs(cdf - uniforms.cpu().numpy()[:, None]).min(axis=-1)


def cdf_rounding_band(
    logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float,
    forbidden_token_ids: Sequence[int] = (), forbidden_token_ids_by_row: torch.Tensor | None = None,
) -> np.ndarray:
    """Per row, the largest gap between the fp32 CDF (the reference's arithmetic,
    one summation order of many) and the exact CDF. Another fp32 summation order
    (a parallel softmax sum over thousands of candidates) lands anywhere inside
    this band, so a uniform closer than it to a boundary may pick either side."""
    cdf, exact = _sampling_cdfs(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                forbidden_token_ids=forbidden_token_ids,
                                forbidden_token_ids_by_row=forbidden_token_ids_by_row)
    return np.abs(cdf - exact).max(axis=-1)
