"""Oracle restatement of the per-op math (TEST INFRASTRUCTURE ONLY).

CPU torch, float32 math with the reference's bf16 rounding points:
* rmsnorm / fused_add_rmsnorm / silu_and_mul follow FlashInfer's kernels as the
  reference calls them (aios/layers/norm.py:10-40, aios/layers/activation.py:9-12):
  fp32 math, one rounding to the storage dtype at the end;
* RoPE is the reference's own bf16 expression (aios/layers/attention.py:6-16) on
  the fp32 cos/sin cache of aios/layers/rotary.py:8-25;
* attention is softmax(q k^T * scale) v in fp32 with the causal cached-prefix mask
  of aios/attention/flashinfer.py:33-91;
* the AttnRes mixer has both the eager (training) form of
  aios/models/minimind_ime.py:27-74 and the single-rounding Triton form of
  aios/kernel/attnres.py:8-127.
"""

from __future__ import annotations

import torch


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    rcp = 1.0 / torch.sqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
    return (xf * rcp * weight.float()).to(x.dtype)


def fused_add_rmsnorm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (normalised x, new residual)."""
    s = x.float() + residual.float()
    rcp = 1.0 / torch.sqrt((s * s).mean(dim=-1, keepdim=True) + eps)
    return (s * rcp * weight.float()).to(x.dtype), s.to(residual.dtype)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    f = x.shape[-1] // 2
    g, u = x[..., :f].float(), x[..., f:].float()
    return (g / (1.0 + torch.exp(-g)) * u).to(x.dtype)


def rope_cache(head_dim: int, max_position: int, base: float) -> tuple[torch.Tensor, torch.Tensor]:
    """aios/layers/rotary.py:13-19 (fp32)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, d]; cos/sin [T, d] fp32 gathered by position; math in x.dtype."""
    c = cos.unsqueeze(1).to(x.dtype)
    s = sin.unsqueeze(1).to(x.dtype)
    return x * c + rotate_half(x) * s


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_positions: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """q [T, Hq, d]; k, v [L, Hkv, d] at key positions 0..L-1; fp32 math.

    Query t attends to keys with position <= q_positions[t]. Returns fp32 [T, Hq, d].
    """
    g = q.shape[1] // k.shape[1]
    kr = k.float().repeat_interleave(g, dim=1)
    vr = v.float().repeat_interleave(g, dim=1)
    scores = torch.einsum("thd,lhd->htl", q.float(), kr) * scale
    key_pos = torch.arange(k.shape[0])
    allowed = key_pos.unsqueeze(0) <= q_positions.unsqueeze(1)
    scores = scores.masked_fill(~allowed.unsqueeze(0), float("-inf"))
    w = scores.softmax(dim=-1)
    return torch.einsum("htl,lhd->thd", w, vr)


def attnres_scores(sources: torch.Tensor, weighted_query: torch.Tensor, eps: float) -> torch.Tensor:
    """aios/models/minimind_ime.py:27-42."""
    sf = sources.float()
    inverse_rms = torch.rsqrt(sf.square().mean(dim=-1) + eps)
    return torch.einsum("d,snd->sn", weighted_query.float(), sf) * inverse_rms


def attnres_mix_eager(
    bank: torch.Tensor, partial: torch.Tensor | None, weighted_query: torch.Tensor, eps: float
) -> torch.Tensor:
    """aios/models/minimind_ime.py:45-74 (training semantics)."""
    if partial is None:
        weights = attnres_scores(bank, weighted_query, eps).softmax(dim=0).to(bank.dtype)
        return torch.einsum("sn,snd->nd", weights, bank)
    bank_logits = attnres_scores(bank, weighted_query, eps)
    pf = partial.float()
    partial_logits = torch.einsum("d,nd->n", weighted_query.float(), pf) * torch.rsqrt(pf.square().mean(-1) + eps)
    weights = torch.cat((bank_logits, partial_logits.unsqueeze(0)), dim=0).softmax(dim=0).to(bank.dtype)
    mixed = torch.einsum("sn,snd->nd", weights[:-1], bank)
    return mixed + weights[-1].unsqueeze(-1) * partial


def attnres_mix_fused(
    bank: torch.Tensor, partial: torch.Tensor | None, weighted_query: torch.Tensor, eps: float
) -> torch.Tensor:
    """aios/kernel/attnres.py:8-127: fp32 scores, bf16 weights, one fp32 sum."""
    sources = bank if partial is None else torch.cat((bank, partial.unsqueeze(0)), dim=0)
    sf = sources.float()
    dot = torch.einsum("d,snd->sn", weighted_query.float(), sf)
    rcp = 1.0 / torch.sqrt(sf.square().mean(-1) + eps)
    w = (dot * rcp).softmax(dim=0).to(bank.dtype).float()
    return torch.einsum("sn,snd->nd", w, sf).to(bank.dtype)
