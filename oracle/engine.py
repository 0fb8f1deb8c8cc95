"""Oracle restatement of one CandidateGroup keystroke (TEST INFRASTRUCTURE ONLY).

Follows aios/ime.py step by step on the CPU:
* _prepare_prefix (1116-1168): token LCP with the previous keystroke, the
  identical-prefix shortcut, backspace => full re-prefill, free the old tail,
  allocate the extension, prefill or extension prefill;
* _generate_branch_batch (891-1054): stateless uniforms per row, min-length and
  refill exact-repeat bans, raw-logprob sampling, EOS/terminal stop codes,
  compaction of finished rows, one decode step per survivor set with slots
  allocated in active-row order (_decode_step, 1219-1251);
* the free-slot FIFO of aios/scheduler/cache.py:9-51 as a Python list.
For page_size 16 the same flow runs on 16-token pages (prefix tokens packed from
page 0; each row's suffix starts on a fresh page).

``run_round(..., forced=...)`` replays a round teacher-forced: at every step the
oracle still draws its own token (recorded as ``own``) but continues with the
forced one, so integer state (slots, page table, stop codes) can be compared bit
for bit and floating-point scores token by token.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import sampler as osamp
from .model import OracleModel, Request


@dataclass
class StepTrace:
    step: int
    rows: list[int]  # local rows sampled at this step (active order)
    own: list[int]  # oracle's own sampled token per row
    tokens: list[int]  # token used (own, or forced)
    logprobs: list[float]  # raw logprob of `tokens` under the oracle logits
    margins: list[float]  # CDF-boundary / top-2 margin of the oracle draw
    slots: list[int] = field(default_factory=list)  # decode slots allocated after this step
    ext_tokens: list[int] | None = None  # draw from external (GPU) logits, if given
    logits: torch.Tensor | None = None  # oracle logits of the active rows


@dataclass
class RoundTrace:
    attempts: int
    row_offset: int
    steps: list[StepTrace]
    output_ids: np.ndarray
    counts: list[int]
    logprob_sums: list[float]
    token_logprobs: np.ndarray
    stop_codes: list[int]
    allocated: list[int]
    active_model_tokens: int


class OracleEngine:
    def __init__(self, model: OracleModel, tokenizer, num_pages: int, page_size: int = 1, table_rows: int = 64,
                 tie_order: str = "index") -> None:
        self.m = model
        self.tok = tokenizer
        self.page_size = page_size
        self.num_pages = num_pages
        self.free = list(range(num_pages))
        self.page_table = np.zeros((table_rows, model.cfg.max_position_embeddings), dtype=np.int64)
        self.tie_order = tie_order
        self.prefix_ids: list[int] = []
        self.prefix_pages: list[int] | None = None
        self.prefix_slots: list[int] | None = None
        self.prefix_logits: torch.Tensor | None = None
        self.terminal_ids = sorted({
            ids[0] for s in "。！？；!?;" if len(ids := tokenizer.encode(s, add_special_tokens=False)) == 1
        })

    # ---- FIFO ------------------------------------------------------------------
    def allocate(self, n: int) -> list[int]:
        if n > len(self.free):
            raise RuntimeError("oracle pool exhausted")
        out, self.free = self.free[:n], self.free[n:]
        return out

    def release(self, ids: list[int]) -> None:
        self.free.extend(ids)

    def _pages_for(self, n: int) -> int:
        return -(-max(0, n) // self.page_size)

    def _slots(self, pages: list[int], start: int, count: int) -> list[int]:
        p = self.page_size
        return [pages[t // p] * p + t % p for t in range(start, start + count)]

    # ---- prefix ------------------------------------------------------------------
    def prepare_prefix(self, token_ids: list[int], table_rows: int) -> tuple[torch.Tensor, list[int], int]:
        self.page_table[:] = 0  # the reference allocates a fresh zero table per keystroke (aios/ime.py:482-485)
        old = self.prefix_ids
        reused = 0
        for a, b in zip(old, token_ids):
            if a != b:
                break
            reused += 1
        n = len(token_ids)
        if self.prefix_pages is not None and self.prefix_logits is not None and reused == len(old) == n:
            self.page_table[:table_rows, :n] = self.prefix_slots
            return self.prefix_logits, self.prefix_pages, reused
        if old and reused == n < len(old):
            reused = 0
        keep = self._pages_for(reused)
        if self.prefix_pages is not None:
            self.release(self.prefix_pages[keep:])
            kept = self.prefix_pages[:keep]
        else:
            kept = []
        pages = kept + self.allocate(self._pages_for(n) - keep)
        slots = pages if self.page_size == 1 else self._slots(pages, 0, n)
        self.page_table[:table_rows, :n] = slots
        req = Request(ids=token_ids[reused:], positions=list(range(reused, n)), new_slots=slots[reused:],
                      key_slots=slots[:n])
        logits = self.m.forward([req])[0]
        self.prefix_ids, self.prefix_pages, self.prefix_slots, self.prefix_logits = list(token_ids), pages, slots, logits
        return logits, pages, reused

    def reset_prefix(self) -> None:
        if self.prefix_pages:
            self.release(self.prefix_pages)
        self.prefix_ids, self.prefix_pages, self.prefix_slots, self.prefix_logits = [], None, None, None

    # ---- one branch batch ------------------------------------------------------
    def run_round(
        self,
        *,
        prefix_logits: torch.Tensor,
        prefix_len: int,
        row_offset: int,
        attempts: int,
        max_new_tokens: int,
        min_new_tokens: int,
        seed: int,
        temperature: float,
        top_k: int,
        top_p: float,
        banned_sequences: list[list[int]] = (),
        ban_min_prefix: int = 2,
        forced: dict | None = None,
        forced_steps: list[list[int]] | None = None,
        external_logits: list[torch.Tensor] | None = None,
    ) -> RoundTrace:
        eos, pad = self.tok.eos_token_id, self.tok.pad_token_id
        S = max_new_tokens
        out_ids = np.full((attempts, S), pad, dtype=np.int64)
        counts = [0] * attempts
        sums = [0.0] * attempts
        tlp = np.zeros((attempts, S), dtype=np.float32)
        stop = [0] * attempts
        uniforms = osamp.stateless_uniforms([seed + r for r in range(attempts)], S)
        minlen = sorted({*self.terminal_ids, eos})
        active = list(range(attempts))
        logits = {r: prefix_logits for r in active}
        row_pages: dict[int, int] = {}
        allocated: list[int] = []
        steps: list[StepTrace] = []
        amt = 0
        width = max((len(s) for s in banned_sequences), default=0)
        for step in range(S):
            by_row = None
            if banned_sequences and step >= ban_min_prefix and step < width:
                by_row = []
                for r in active:
                    ids = []
                    for seq in banned_sequences:
                        match = len(seq) > step and list(out_ids[r, :step]) == list(seq[:step])
                        ids.append(seq[step] if match else pad)
                    by_row.append(ids)
                by_row = torch.tensor(by_row)
            batch_logits = torch.stack([logits[r] for r in active])
            ext = None
            if external_logits is not None:
                # also draw from logits produced elsewhere (the GPU's, same step and
                # rows), to check the sampling + bookkeeping logic bit for bit
                ext = external_logits[step][active].to(torch.bfloat16)
            u = uniforms[active, step]
            own, lp_own = osamp.sample_with_logprobs(
                batch_logits, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u,
                forbidden_token_ids=minlen if step < min_new_tokens else (), forbidden_token_ids_by_row=by_row,
                tie_order=self.tie_order,
            )
            own = own.squeeze(-1).tolist()
            ext_tokens = None
            if ext is not None:
                et, _ = osamp.sample_with_logprobs(
                    ext, temperature=temperature, top_k=top_k, top_p=top_p, uniforms=u,
                    forbidden_token_ids=minlen if step < min_new_tokens else (), forbidden_token_ids_by_row=by_row,
                    tie_order=self.tie_order,
                )
                ext_tokens = et.squeeze(-1).tolist()
            raw = torch.log_softmax(batch_logits.float(), dim=-1)
            if osamp.is_greedy(temperature, top_k, top_p):
                top2 = batch_logits.float().topk(2, dim=-1).values
                margins = (top2[:, 0] - top2[:, 1]).tolist()
            else:
                margins = osamp.sample_margin(batch_logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                              uniforms=u, forbidden_token_ids=minlen if step < min_new_tokens else (),
                                              forbidden_token_ids_by_row=by_row).tolist()
            toks = list(own)
            if forced is not None:
                for i, r in enumerate(active):
                    toks[i] = forced_token(forced, r, step, eos)
            elif forced_steps is not None:
                toks = list(forced_steps[step])  # tokens of the active rows, in active order
            lps = [float(raw[i, t]) for i, t in enumerate(toks)]
            trace = StepTrace(step=step, rows=list(active), own=own, tokens=toks, logprobs=lps, margins=margins,
                              ext_tokens=ext_tokens, logits=batch_logits)
            steps.append(trace)
            finished = []
            for i, r in enumerate(active):
                t = toks[i]
                is_eos = t == eos
                if not is_eos:
                    out_ids[r, step] = t
                    counts[r] += 1
                    sums[r] = float(np.float32(sums[r]) + np.float32(lps[i]))
                    tlp[r, step] = lps[i]
                terminal = (not is_eos) and t in self.terminal_ids
                if is_eos:
                    stop[r] = 1
                if terminal:
                    stop[r] = 2
                finished.append(is_eos or terminal)
            if step + 1 == S:
                break
            survivors = [r for i, r in enumerate(active) if not finished[i]]
            survivor_tokens = [toks[i] for i, r in enumerate(active) if not finished[i]]
            active = survivors
            if not active:
                break
            amt += len(active)
            pos = prefix_len + step
            reqs, slots = [], []
            if self.page_size == 1:
                new = self.allocate(len(active))
                allocated += new
                slots = new
            else:
                if step % self.page_size == 0:
                    new = self.allocate(len(active))
                    allocated += new
                    for r, pg in zip(active, new):
                        row_pages[r] = pg
                slots = [row_pages[r] * self.page_size + step % self.page_size for r in active]
            trace.slots = slots
            for r, t, s in zip(active, survivor_tokens, slots):
                self.page_table[row_offset + r, pos] = s
                reqs.append(Request(ids=[t], positions=[pos], new_slots=[s],
                                    key_slots=[int(x) for x in self.page_table[row_offset + r, : pos + 1]]))
            out = self.m.forward(reqs)
            logits = {r: out[i] for i, r in enumerate(active)}
        return RoundTrace(attempts=attempts, row_offset=row_offset, steps=steps, output_ids=out_ids, counts=counts,
                          logprob_sums=sums, token_logprobs=tlp, stop_codes=stop, allocated=allocated,
                          active_model_tokens=amt)


def forced_token(forced: dict, row: int, step: int, eos: int) -> int:
    """Token a recorded round emitted at (row, step): the emitted id, or EOS at
    the step that stopped the row with stop code 1."""
    counts = forced["counts"]
    if step < counts[row]:
        return int(forced["output_ids"][row][step])
    if forced["stop_codes"][row] == 1 and step == counts[row]:
        return eos
    raise ValueError(f"row {row} produced no token at step {step}")
