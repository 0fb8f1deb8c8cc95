"""IME CandidateGroup engine (replaces aios/ime.py:373-1251).

``ImeCompletionEngine.complete(prefix, config, cancellation)`` keeps the
reference's API and result fields: token-LCP reuse of the previous keystroke's
prefix KV, one prefix (re-)prefill, lock-step decode of N candidate rows sharing
the prefix KV, raw-logprob scoring, host text filters and MMR Top-3, adaptive
refill rounds, latest-wins cancellation. The per-token loop runs on the device
(``runtime.group``); the host launches one CUDA graph per step and reads the
round's results back once.
"""

from __future__ import annotations

import math
import threading
import time
from typing import Literal

import numpy as np
import torch

from .core import Batch, Req, SamplingParams
from .ime_text import (  # noqa: F401  (re-exported public names)
    ASSISTANT_PATTERN,
    FUNCTION_WORD_ENDINGS,
    NATURAL_REDUPLICATIONS,
    REPEAT_PATTERN,
    TERMINAL_TEXT_PATTERN,
    CandidatePoolStats,
    ImeCandidate,
    ImeCandidateScore,
    ImeCompletionResult,
    ImeGenerationConfig,
    ImeScoringResult,
    adaptive_refill_attempts,
    candidate_key,
    candidate_pool_stats,
    invalid_reasons,
    ngram_similarity,
    normalize_candidate,
    repeated_ngram,
    select_top_candidates,
    soft_penalty,
    token_longest_common_prefix,
    truncate_at_terminal,
)
from .kernel import ops
from .runtime.group import CandidateGroupRuntime, RoundResult
from .runtime.prefill import PrefixRunner

TERMINAL_SYMBOLS = "。！？；!?;"


class CancellationToken:
    """Latest-wins cancellation (aios/ime.py:174-184). ``cancel()`` also writes
    every host-mapped device flag attached to the token, so a round already
    running on the GPU stops at its next step boundary."""

    def __init__(self, generation_id: int) -> None:
        self.generation_id = generation_id
        self._event = threading.Event()
        self._flags: list[torch.Tensor] = []
        self._lock = threading.Lock()

    def cancel(self) -> None:
        with self._lock:
            self._event.set()
            for flag in self._flags:
                flag.numpy()[0] = 1

    @property
    def cancelled(self) -> bool:
        return self._event.is_set()

    def _attach_flag(self, flag: torch.Tensor) -> None:
        with self._lock:
            self._flags.append(flag)
            if self._event.is_set():
                flag.numpy()[0] = 1

    def _detach_flag(self, flag: torch.Tensor) -> None:
        with self._lock:
            self._flags = [f for f in self._flags if f is not flag]


class ImeCompletionEngine:
    """Single-user, same-prefix candidate-group runtime for MiniMind-IME."""

    MAX_TABLE_ROWS = 64

    def __init__(self, llm) -> None:
        self.llm = llm
        self._generation_id = 0
        self._active_token: CancellationToken | None = None
        self._generation_lock = threading.Lock()
        self._run_lock = threading.Lock()
        self._prefix_token_ids: list[int] = []
        self._prefix_pages: list[int] | None = None
        self._prefix_slots: list[int] | None = None
        self._prefix_logits: torch.Tensor | None = None
        self.page_size = llm.cache_manager.page_size
        self._page_table = torch.zeros(
            (self.MAX_TABLE_ROWS, llm.config.max_position_embeddings), dtype=torch.int32, device=llm.device
        )
        llm.ctx.page_table = self._page_table
        self._terminal_token_ids = {
            ids[0]
            for symbol in TERMINAL_SYMBOLS
            if len(ids := llm.tokenizer.encode(symbol, add_special_tokens=False)) == 1
        }
        self._terminal_list = sorted(self._terminal_token_ids)
        eos = llm.tokenizer.eos_token_id
        self._minlen_ids = sorted({*self._terminal_token_ids, *((eos,) if eos is not None else ())})
        self._runtime = CandidateGroupRuntime(llm)
        self._prefix_runner = PrefixRunner(llm)

    # ------------------------------------------------------------------ API
    def new_generation(self) -> CancellationToken:
        with self._generation_lock:
            if self._active_token is not None:
                self._active_token.cancel()
            self._generation_id += 1
            self._active_token = CancellationToken(self._generation_id)
            return self._active_token

    def reset_prefix_cache(self) -> None:
        """Release the persistent single-user prefix KV pages."""
        with self._run_lock:
            self._reset_prefix_cache_unlocked()

    def _reset_prefix_cache_unlocked(self) -> None:
        if self._prefix_pages:
            self.llm.cache_manager.give(self._prefix_pages)
        self._prefix_token_ids = []
        self._prefix_pages = None
        self._prefix_slots = None
        self._prefix_logits = None

    @torch.inference_mode()
    def complete(
        self,
        prefix: str,
        config: ImeGenerationConfig | None = None,
        cancellation: CancellationToken | None = None,
    ) -> ImeCompletionResult:
        cancellation = cancellation or self.new_generation()
        with self._run_lock:
            return self._complete_locked(prefix, config, cancellation)

    # ------------------------------------------------------------------ helpers
    def _pages_for(self, tokens: int) -> int:
        return -(-max(0, tokens) // self.page_size)

    def _encode_prefix(self, prefix: str) -> list[int]:
        token_ids = self.llm.tokenizer.encode(prefix, add_special_tokens=False)
        if self.llm.tokenizer.bos_token_id is not None:
            token_ids = [self.llm.tokenizer.bos_token_id, *token_ids]
        if not token_ids:
            raise ValueError("prefix produced no input tokens")
        return token_ids

    def _cancelled_result(self, prefix, token_ids, cancellation, wall_started) -> ImeCompletionResult:
        return ImeCompletionResult(
            prefix=prefix, generation_id=cancellation.generation_id, cancelled=True, candidates=(),
            raw_candidates=(), prefix_tokens=len(token_ids), sampling_attempts=0, generated_tokens=0,
            active_model_tokens=0, latency_ms=(time.perf_counter() - wall_started) * 1000.0, gpu_latency_ms=0.0,
            unique_kv_pages=0, reused_prefix_tokens=0, refill_rounds=0, valid_unique_candidates=0,
            invalid_candidates=0, duplicate_candidates=0, refill_stop_reason="cancelled",
        )

    def _forbidden_sequences(self, raw_candidates: list[ImeCandidate], config: ImeGenerationConfig) -> list[list[int]]:
        """Exact-repeat bans for a refill round (aios/ime.py:537-556)."""
        out: list[list[int]] = []
        if not config.refill_avoid_exact_repeats:
            return out
        seen: set[str] = set()
        for cand in sorted(raw_candidates, key=lambda item: item.base_score, reverse=True):
            key = candidate_key(cand.text)
            if not key or key in seen:
                continue
            seq = self.llm.tokenizer.encode(cand.text, add_special_tokens=False)
            if len(seq) > config.refill_ban_min_prefix_tokens:
                out.append(seq)
                seen.add(key)
        return out

    # ------------------------------------------------------------------ keystroke
    def _complete_locked(
        self, prefix: str, config: ImeGenerationConfig | None, cancellation: CancellationToken
    ) -> ImeCompletionResult:
        wall_started = time.perf_counter()
        config = config or ImeGenerationConfig()
        config.validate()
        token_ids = self._encode_prefix(prefix)
        if cancellation.cancelled:
            return self._cancelled_result(prefix, token_ids, cancellation, wall_started)
        max_total_len = len(token_ids) + config.max_new_tokens
        if max_total_len > self.llm.config.max_position_embeddings:
            raise ValueError(
                f"prefix + output exceeds context limit: {max_total_len} > {self.llm.config.max_position_embeddings}"
            )
        max_concurrent = max(config.sampling_attempts, config.refill_batch_size)
        required_pages = self._pages_for(len(token_ids)) + max_concurrent * self._pages_for(config.max_new_tokens - 1)
        if required_pages > self.llm.num_pages:
            raise ValueError(
                "IME CandidateGroup KV budget is too small: "
                f"need up to {required_pages} pages, configured {self.llm.num_pages}; "
                "increase kv_cache_max_tokens or shorten the context/output"
            )
        max_attempts = config.max_sampling_attempts
        if max_attempts > self.MAX_TABLE_ROWS or max_concurrent > self._runtime.max_rows:
            raise ValueError(
                f"at most {self.MAX_TABLE_ROWS} attempts per keystroke and {self._runtime.max_rows} per round"
            )
        if config.max_new_tokens > self._runtime.max_steps:
            raise ValueError(f"max_new_tokens above {self._runtime.max_steps}")
        started = torch.cuda.Event(enable_timing=True)
        ended = torch.cuda.Event(enable_timing=True)
        started.record()
        cancelled = False
        cm = self.llm.cache_manager
        # rows [0, max_attempts) are reset to the prefix + zeros, like the fresh
        # table the reference allocates per keystroke (aios/ime.py:482-485)
        prefix_logits, prefix_pages, reused = self._prepare_prefix(token_ids, max_attempts, max_total_len)
        peak_unique_pages = len(prefix_pages)
        raw_candidates: list[ImeCandidate] = []
        actual_attempts = 0
        generated_tokens = 0
        active_model_tokens = len(token_ids) - reused
        refill_rounds = 0
        refill_stop_reason = "max_attempts"
        selected: list[ImeCandidate] = []
        while actual_attempts < max_attempts:
            if actual_attempts == 0:
                attempts = config.sampling_attempts
                temperature, top_k, top_p = config.temperature, config.top_k, config.top_p
                forbidden: list[list[int]] = []
            else:
                elapsed_ms = (time.perf_counter() - wall_started) * 1000.0
                if config.refill_deadline_ms > 0.0 and elapsed_ms >= config.refill_deadline_ms:
                    refill_stop_reason = "deadline"
                    break
                attempts = adaptive_refill_attempts(raw_candidates, config, actual_attempts)
                if attempts == 0:
                    refill_stop_reason = "filled"
                    break
                refill_rounds += 1
                temperature, top_k, top_p = config.refill_schedule(refill_rounds)
                forbidden = self._forbidden_sequences(raw_candidates, config)
            head_before = cm.head
            result = self._runtime.run_round(
                prefix_logits=prefix_logits, prefix_len=len(token_ids), row_offset=actual_attempts,
                attempts=attempts, max_new_tokens=config.max_new_tokens, min_new_tokens=config.min_new_tokens,
                seed=config.seed + actual_attempts * 100_003, temperature=temperature, top_k=top_k, top_p=top_p,
                terminal_ids=self._terminal_list, minlen_ids=self._minlen_ids, banned_sequences=forbidden,
                ban_min_prefix=config.refill_ban_min_prefix_tokens, eos_id=self.llm.tokenizer.eos_token_id,
                pad_id=self.llm.tokenizer.pad_token_id, cancellation=cancellation,
            )
            raw_candidates.extend(self._candidates_from(result, prefix, config))
            peak_unique_pages = max(peak_unique_pages, len(prefix_pages) + result.pages_consumed)
            actual_attempts += attempts
            generated_tokens += sum(result.counts)
            active_model_tokens += result.active_model_tokens
            cancelled |= result.cancelled
            # candidate text is materialised: the round's suffix KV goes back to the FIFO
            cm.free_range(head_before, result.pages_consumed)
            selected = select_top_candidates(raw_candidates, config.display_candidates, config.diversity_lambda)
            if cancelled or len(selected) >= config.display_candidates:
                refill_stop_reason = "cancelled" if cancelled else "filled"
                break
        ended.record()
        ended.synchronize()
        gpu_latency_ms = started.elapsed_time(ended)
        # `selected` was computed after the last round was added (the loop only
        # leaves before adding a round when the refill deadline or budget ends it)
        stats = candidate_pool_stats(raw_candidates)
        if (
            refill_stop_reason == "max_attempts"
            and actual_attempts < max_attempts
            and len(selected) >= config.display_candidates
        ):
            refill_stop_reason = "filled"
        return ImeCompletionResult(
            prefix=prefix,
            generation_id=cancellation.generation_id,
            cancelled=cancelled,
            candidates=tuple(selected),
            raw_candidates=tuple(raw_candidates),
            prefix_tokens=len(token_ids),
            sampling_attempts=actual_attempts,
            generated_tokens=generated_tokens,
            active_model_tokens=active_model_tokens,
            latency_ms=(time.perf_counter() - wall_started) * 1000.0,
            gpu_latency_ms=gpu_latency_ms,
            unique_kv_pages=peak_unique_pages,
            reused_prefix_tokens=reused,
            refill_rounds=refill_rounds,
            valid_unique_candidates=stats.valid_unique_candidates,
            invalid_candidates=stats.invalid_candidates,
            duplicate_candidates=stats.duplicate_candidates,
            refill_stop_reason=refill_stop_reason,
        )

    def _candidates_from(self, result: RoundResult, prefix: str, config: ImeGenerationConfig) -> list[ImeCandidate]:
        """Text post-processing of one round (aios/ime.py:1056-1107)."""
        tok = self.llm.tokenizer
        rows = [result.output_ids[r, : result.counts[r]].tolist() for r in range(len(result.counts))]
        decoded = tok.batch_decode(rows, skip_special_tokens=True, clean_up_tokenization_spaces=False)
        out: list[ImeCandidate] = []
        for r, text in enumerate(decoded):
            normalized, decoded_terminal = truncate_at_terminal(normalize_candidate(text))
            count = result.counts[r]
            score_sum = result.logprob_sums[r]
            if decoded_terminal and result.stop_codes[r] == 0:
                # a token holding both a terminator and more text: score only up to
                # the first token whose decoded prefix contains the terminator
                for consumed in range(1, count + 1):
                    partial = tok.decode(rows[r][:consumed], skip_special_tokens=True,
                                         clean_up_tokenization_spaces=False)
                    if TERMINAL_TEXT_PATTERN.search(normalize_candidate(partial)):
                        count = consumed
                        score_sum = float(np.float32(result.token_logprobs[r, :consumed].sum(dtype=np.float32)))
                        break
            reasons = invalid_reasons(normalized, config, prefix)
            average = score_sum / count if count else float("-inf")
            score = average - soft_penalty(normalized) if not reasons else float("-inf")
            stop_reason = {1: "eos", 2: "terminal_punctuation"}.get(
                result.stop_codes[r], "decoded_terminal" if decoded_terminal else "max_new_tokens"
            )
            out.append(ImeCandidate(
                text=normalized, token_count=count, average_logprob=average, base_score=score,
                selection_score=score, stop_reason=stop_reason, invalid_reasons=reasons,
            ))
        return out

    # ------------------------------------------------------------------ prefix
    def _slots_for_pages(self, pages: list[int], count: int) -> list[int]:
        """Token slots [0, count) of a prefix laid out on `pages` (page_size slots each)."""
        p = self.page_size
        if p == 1:
            return list(pages[:count])
        return [pages[t // p] * p + t % p for t in range(count)]

    def _prepare_prefix(self, token_ids: list[int], table_rows: int, width: int) -> tuple[torch.Tensor, list[int], int]:
        """Build or incrementally extend the persistent latest-prefix KV
        (aios/ime.py:1116-1168); resets page-table rows [0, table_rows) to the
        prefix (zeros up to `width`); returns (logits [1, V], prefix pages, reused).
        Slot ids are known on the host (the FIFO has an exact host mirror), so the
        prefill inputs travel in one copy and the forward replays as a CUDA graph."""
        cm = self.llm.cache_manager
        old_ids = self._prefix_token_ids
        old_pages = self._prefix_pages
        reused = token_longest_common_prefix(old_ids, token_ids)
        n = len(token_ids)
        if old_pages is not None and self._prefix_logits is not None and reused == len(old_ids) == n:
            self._prefix_runner.fill_table(self._page_table, table_rows, width, n)
            return self._prefix_logits, old_pages, reused
        # Backspace only: the old cache holds no logits at the new last token.
        if old_ids and reused == n < len(old_ids):
            reused = 0
        keep_pages = self._pages_for(reused)
        kept: list[int] = []
        if old_pages is not None:
            kept = old_pages[:keep_pages]
            if len(old_pages) > keep_pages:
                cm.give(old_pages[keep_pages:])
        prefix_pages = kept + cm.take(self._pages_for(n) - keep_pages)
        prefix_slots = self._slots_for_pages(prefix_pages, n)
        logits = self._prefix_runner.run(token_ids, reused, prefix_slots, self._page_table, table_rows, width)
        self._prefix_token_ids = list(token_ids)
        self._prefix_pages = prefix_pages
        self._prefix_slots = prefix_slots
        self._prefix_logits = logits
        return logits, prefix_pages, reused

    # ------------------------------------------------------------------ scoring
    @torch.inference_mode()
    def score_candidates(
        self, prefix: str, candidates: list[str], mode: Literal["stable", "shared_decode"] = "stable"
    ) -> ImeScoringResult:
        """Teacher-force and rank a candidate group by raw average LM score
        (aios/ime.py:642-889)."""
        if not candidates:
            raise ValueError("candidates must not be empty")
        with self._run_lock:
            if mode == "stable":
                return self._score_stable_locked(prefix, candidates)
            if mode == "shared_decode":
                return self._score_shared_locked(prefix, candidates)
            raise ValueError(f"Unsupported scoring mode: {mode}")

    def _score_stable_locked(self, prefix: str, candidates: list[str]) -> ImeScoringResult:
        wall_started = time.perf_counter()
        tok = self.llm.tokenizer
        prefix_ids = self._encode_prefix(prefix)
        cand_ids = [tok.encode(text, add_special_tokens=False) for text in candidates]
        sequences = [[*prefix_ids, *ids] for ids in cand_ids]
        max_total = max(map(len, sequences))
        if max_total > self.llm.config.max_position_embeddings:
            raise ValueError(
                f"prefix + candidate exceeds context limit: {max_total} > {self.llm.config.max_position_embeddings}"
            )
        if len(candidates) > self.MAX_TABLE_ROWS:
            raise ValueError(f"at most {self.MAX_TABLE_ROWS} candidates per call")
        self._reset_prefix_cache_unlocked()
        required = sum(self._pages_for(len(s)) for s in sequences)
        if required > self.llm.num_pages:
            raise ValueError(
                f"Stable candidate scoring KV budget is too small: need {required} pages, configured {self.llm.num_pages}"
            )
        dev = self.llm.device
        cm = self.llm.cache_manager
        started = torch.cuda.Event(enable_timing=True)
        ended = torch.cuda.Event(enable_timing=True)
        started.record()
        allocated: list[int] = []
        try:
            reqs, slots = [], []
            table_rows = torch.zeros((len(sequences), max_total), dtype=torch.int32)
            for row, seq in enumerate(sequences):
                pages = cm.take(self._pages_for(len(seq)))
                allocated += pages
                s = self._slots_for_pages(pages, len(seq))
                table_rows[row, : len(seq)] = torch.tensor(s, dtype=torch.int32)
                slots += s
                reqs.append(Req(input_ids=torch.empty(len(seq), dtype=torch.long), cached_len=0, output_len=1,
                                uid=row, sampling_params=SamplingParams(max_tokens=1), table_idx=row))
            self._page_table[: len(sequences), :max_total].copy_(table_rows.pin_memory(), non_blocking=True)
            batch = Batch(reqs=reqs, phase="prefill", return_all_logits=True)
            flat = [t for s in sequences for t in s]
            pos = [i for s in sequences for i in range(len(s))]
            staged = torch.tensor(flat + pos + slots, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            batch.input_ids = staged[: len(flat)]
            batch.positions = staged[len(flat) : 2 * len(flat)]
            batch.out_loc = staged[2 * len(flat) :]
            self.llm.model.attn_backend.prepare_metadata(batch)
            with self.llm.ctx.forward_batch(batch):
                logits = self.llm.model.forward()
            rows, targets, owners = [], [], []
            offset = 0
            for i, (seq, ids) in enumerate(zip(sequences, cand_ids)):
                for j, t in enumerate(ids):
                    rows.append(offset + len(prefix_ids) - 1 + j)
                    targets.append(t)
                    owners.append(i)
                offset += len(seq)
            lp = ops.token_logprobs(logits.index_select(0, torch.tensor(rows, device=dev)),
                                    torch.tensor(targets, device=dev)) if rows else None
            ended.record()
            ended.synchronize()
            lp_host = lp.cpu().numpy() if lp is not None else np.zeros(0, np.float32)
            scored = []
            for i, (text, ids) in enumerate(zip(candidates, cand_ids)):
                vals = lp_host[[k for k, o in enumerate(owners) if o == i]]
                if ids:
                    total = float(np.float32(vals.sum(dtype=np.float32)))
                    scored.append(ImeCandidateScore(text=text, token_count=len(ids),
                                                    average_logprob=float(np.float32(vals.mean(dtype=np.float32))),
                                                    sum_logprob=total))
                else:
                    scored.append(ImeCandidateScore(text=text, token_count=0, average_logprob=float("-inf"),
                                                    sum_logprob=float("-inf")))
            scored.sort(key=lambda item: item.average_logprob, reverse=True)
            return ImeScoringResult(
                prefix=prefix, candidates=tuple(scored), latency_ms=(time.perf_counter() - wall_started) * 1000.0,
                gpu_latency_ms=started.elapsed_time(ended), unique_kv_pages=len(allocated),
                reused_prefix_tokens=0,
            )
        finally:
            if allocated:
                cm.give(allocated)

    def _score_shared_locked(self, prefix: str, candidates: list[str]) -> ImeScoringResult:
        wall_started = time.perf_counter()
        tok = self.llm.tokenizer
        prefix_ids = self._encode_prefix(prefix)
        cand_ids = [tok.encode(text, add_special_tokens=False) for text in candidates]
        max_cand = max((len(ids) for ids in cand_ids), default=0)
        max_total = len(prefix_ids) + max_cand
        if max_total > self.llm.config.max_position_embeddings:
            raise ValueError(
                f"prefix + candidate exceeds context limit: {max_total} > {self.llm.config.max_position_embeddings}"
            )
        if self.page_size != 1:
            raise ValueError("shared-decode scoring runs on a page_size=1 pool")
        required = len(prefix_ids) + len(candidates) * max(0, max_cand - 1)
        if required > self.llm.num_pages:
            raise ValueError(
                f"Shared-decode scoring KV budget is too small: need up to {required} pages, configured {self.llm.num_pages}"
            )
        if len(candidates) > self.MAX_TABLE_ROWS:
            raise ValueError(f"at most {self.MAX_TABLE_ROWS} candidates per call")
        dev = self.llm.device
        cm = self.llm.cache_manager
        started = torch.cuda.Event(enable_timing=True)
        ended = torch.cuda.Event(enable_timing=True)
        started.record()
        allocated: list[int] = []
        try:
            prefix_logits, prefix_pages, reused = self._prepare_prefix(prefix_ids, len(candidates), max_total)
            sums = torch.zeros(len(candidates), dtype=torch.float32, device=dev)
            first = [i for i, ids in enumerate(cand_ids) if ids]
            if first:
                lp = ops.token_logprobs(prefix_logits.expand(len(first), -1),
                                        torch.tensor([cand_ids[i][0] for i in first], device=dev))
                sums.index_add_(0, torch.tensor(first, device=dev), lp)
            for step in range(1, max_cand):
                active = [i for i, ids in enumerate(cand_ids) if len(ids) > step]
                if not active:
                    break
                cached_len = len(prefix_ids) + step - 1
                pages = cm.take(len(active))
                allocated += pages
                reqs = [Req(input_ids=torch.empty(cached_len + 1, dtype=torch.long), cached_len=cached_len,
                            output_len=1, uid=i, sampling_params=SamplingParams(max_tokens=1), table_idx=i)
                        for i in active]
                batch = Batch(reqs=reqs, phase="decode")
                host = [cand_ids[i][step - 1] for i in active] + [cached_len] * len(active) + pages + active
                staged = torch.tensor(host, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
                n_act = len(active)
                batch.input_ids = staged[:n_act]
                batch.positions = staged[n_act : 2 * n_act]
                batch.out_loc = staged[2 * n_act : 3 * n_act]
                self._page_table[staged[3 * n_act :].long(), cached_len] = batch.out_loc
                self.llm.model.attn_backend.prepare_metadata(batch)
                with self.llm.ctx.forward_batch(batch):
                    logits = self.llm.model.forward()
                lp = ops.token_logprobs(logits, torch.tensor([cand_ids[i][step] for i in active], device=dev))
                sums.index_add_(0, torch.tensor(active, device=dev), lp)
            ended.record()
            ended.synchronize()
            totals = sums.cpu().tolist()
            scored = [
                ImeCandidateScore(text=text, token_count=len(ids),
                                  average_logprob=(total / len(ids) if ids else float("-inf")),
                                  sum_logprob=(total if ids else float("-inf")))
                for text, ids, total in zip(candidates, cand_ids, totals)
            ]
            scored.sort(key=lambda item: item.average_logprob, reverse=True)
            return ImeScoringResult(
                prefix=prefix, candidates=tuple(scored), latency_ms=(time.perf_counter() - wall_started) * 1000.0,
                gpu_latency_ms=started.elapsed_time(ended),
                unique_kv_pages=len(prefix_pages) + len(allocated), reused_prefix_tokens=reused,
            )
        finally:
            if allocated:
                cm.give(allocated)
