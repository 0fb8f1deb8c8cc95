"""Sampler (replaces aios/engine/sample.py:12-167) on the sm_100a sampling kernel.

``sample_with_logprobs`` keeps the reference's signature, argument checks and
contract: tokens are drawn from the temperature / top-k / top-p distribution of
the logits with forbidden ids removed, while the returned score is the raw
log-probability under the unmodified model distribution. ``uniforms`` gives
request-local stateless sampling (inverse CDF); without it the uniforms are drawn
from ``generator`` (torch.rand), the same distribution as the reference's
multinomial draw. Equal logits are ordered by ascending token id.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from ..core import SamplingParams
from ..kernel import ops

MASK64 = (1 << 64) - 1


def _as_int64(seed: int) -> int:
    value = int(seed) & MASK64
    return value - (1 << 64) if value >= (1 << 63) else value


def stateless_uniforms(candidate_seeds: Sequence[int], steps: int, device: torch.device) -> torch.Tensor:
    """[rows, steps] uniforms keyed by (candidate_seed, token_step): a surviving
    candidate draws the same continuation whatever rows finished before it."""
    if steps < 1:
        raise ValueError("steps must be positive")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("stateless_uniforms runs on a CUDA device")
    seeds = torch.tensor([_as_int64(s) for s in candidate_seeds], dtype=torch.int64)
    if seeds.numel() == 0:
        return torch.empty((0, steps), dtype=torch.float32, device=device)
    return ops.stateless_uniforms_device(seeds.pin_memory().to(device, non_blocking=True), steps)


@dataclass
class Sampler:
    sampling_params: SamplingParams

    def sample_with_logprobs(
        self,
        logits: torch.Tensor,
        *,
        generator: torch.Generator | None = None,
        uniforms: torch.Tensor | None = None,
        forbidden_token_ids: Sequence[int] = (),
        forbidden_token_ids_by_row: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        if generator is not None and uniforms is not None:
            raise ValueError("generator and uniforms are mutually exclusive")
        if not logits.is_cuda:
            raise ValueError("Sampler runs on CUDA logits")
        squeeze = logits.ndim == 1
        logits2 = logits.unsqueeze(0) if squeeze else logits
        if logits2.ndim != 2:
            raise ValueError("logits must have shape [batch, vocab] or [vocab]")
        if logits2.stride(-1) != 1:
            logits2 = logits2.contiguous()
        if logits2.dtype != torch.bfloat16:
            logits2 = logits2.to(torch.bfloat16)
        rows, vocab = logits2.shape
        dev = logits2.device
        forbidden = None
        if forbidden_token_ids:
            blocked = sorted({int(t) for t in forbidden_token_ids})
            invalid = [t for t in blocked if t < 0 or t >= vocab]
            if invalid:
                raise ValueError(f"forbidden token ids are outside the vocabulary: {invalid}")
            forbidden = torch.tensor(blocked, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        by_row = None
        if forbidden_token_ids_by_row is not None:
            if logits.ndim != 2:
                raise ValueError("row-specific forbidden ids require 2D logits")
            if forbidden_token_ids_by_row.ndim != 2 or forbidden_token_ids_by_row.shape[0] != rows:
                raise ValueError("forbidden_token_ids_by_row must have shape [batch, count]")
            if forbidden_token_ids_by_row.device.type == "cpu" and not bool(
                ((forbidden_token_ids_by_row >= 0) & (forbidden_token_ids_by_row < vocab)).all().item()
            ):
                raise ValueError("row-specific forbidden token ids are outside the vocabulary")
            by_row = forbidden_token_ids_by_row.to(device=dev, dtype=torch.int64).contiguous()
            if by_row.shape[1] == 0:
                by_row = None
        sp = self.sampling_params
        greedy = sp.is_greedy
        u = None
        if not greedy:
            if uniforms is None:
                u = torch.rand(rows, generator=generator, dtype=torch.float32,
                               device=generator.device if generator is not None else dev).to(dev)
            else:
                if tuple(uniforms.shape) != (rows,) and not (squeeze and uniforms.numel() == 1):
                    raise ValueError(
                        "uniforms must match the sampling batch dimensions: "
                        f"expected {tuple(logits.shape[:-1])}, got {tuple(uniforms.shape)}"
                    )
                u = uniforms.reshape(rows).to(device=dev, dtype=torch.float32).contiguous()
        tok, lp = ops.sample(
            logits2, temperature=sp.temperature if not greedy else 1.0, top_k=sp.top_k, top_p=sp.top_p,
            greedy=greedy, uniforms=u, forbidden=forbidden, forbidden_rows=by_row,
        )
        if squeeze:
            return tok[0], lp[0]
        return tok, lp

    def sample(self, logits: torch.Tensor) -> torch.Tensor:
        return self.sample_with_logprobs(logits)[0]
