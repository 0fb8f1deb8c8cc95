"""CandidateGroup branch-batch runtime: the device-side replacement of
``ImeCompletionEngine._generate_branch_batch``'s step loop (aios/ime.py:891-1054).

One round of ``attempts`` candidate rows runs as

    group_begin                      (reset rows, broadcast prefix logits, uniforms)
    group_step                       (first sample, from the prefix row)
    [decode forward + group_step] x (max_new_tokens - 1)   (one CUDA graph replay each)

Inside a step graph the step follows the forward's LM head and reads its state
before waiting on it (AIOSB_GROUP_AFTER_FORWARD); the LM head leaves one SM per
row free so that the step's CTAs start while it runs.

``group_step`` samples every active row, does the EOS/terminal bookkeeping,
compacts finished rows and allocates the next KV slots from the device FIFO in
active-row order, then writes the decode forward's ids / positions / slots; the
forward (every layer's kernels) reads them from fixed device buffers, so the
whole step is one graph replay with no host round trip. Finished rows stay in
their slot but are masked out (no KV write, no attention), which keeps each
row's outputs identical to the reference's compacted batch.

The host never synchronises inside a round: it keeps at most two steps queued
ahead of the device by polling a host-mapped progress word, stops launching once
the device reports the group done, and reads all results back with one event
wait at the end. Cancellation is observed by the device between steps through a
host-mapped flag that ``CancellationToken.cancel`` writes.
"""

from __future__ import annotations

import ctypes
import os
import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from ..attention import B200AttentionMetadata
from ..core import Batch, Req, SamplingParams
from ..kernel import ops

MAX_TERMINAL = 16
MAX_MINLEN = 32
SORT_K = 2048  # sorted candidates of the step kernel's top-k path
LARGE_SORT_VOCAB = 16384  # larger sorted sets sort whole rows: vocabularies up to this size

# The persistent decode step (one launch per decode forward, aiosb_decode_step)
# serves the standard-residual models with these dims when
# AIOSB_PERSISTENT_DECODE=1. The default is the per-kernel forward: on B200 its
# chain of programmatic-dependent launches (about 2.5 us per linear) beats the
# persistent kernel's cross-CTA exchanges through L2 (measured 326-405 us per
# S10 step against about 220 us). Both are complete forwards with the same
# rounding points.
_PERSISTENT = os.environ.get("AIOSB_PERSISTENT_DECODE", "0") == "1"

# How the decode attention reads its key history (aiosb_attention_decode's
# stable_history): "staged" (every row's CTA reads its keys itself, before the
# dependency wait), "prefix_once" (the rows of a KV head split the shared prefix
# and exchange it over distributed shared memory, before the wait) or "cascade"
# (the cluster-cascade kernel, everything after the wait).
HISTORY_MODES = {"cascade": 0, "staged": _lib.HISTORY_STAGED, "prefix_once": _lib.HISTORY_PREFIX_ONCE}
_HISTORY = HISTORY_MODES[os.environ.get("AIOSB_DECODE_HISTORY", "staged")]
# Prefix lengths up to which the decode attention stages the whole prefix before
# its dependency wait, one step graph per class: its shared memory grows with the
# class (a 512-key class costs every short keystroke about 2-5%).
STAGE_CLASSES = (128, 512)


# Sampling from the LM head's tile statistics (aiosb_group_ptrs.tile_stats): the
# decode forward's LM head also writes, per 16-id tile of each row, the max, the
# sum of exponentials, the min and a NaN flag, and the step kernel bounds its
# top-k candidates and the log-sum-exp from those instead of scanning the row.
# AIOSB_TILE_SAMPLING=0 keeps the row scan.
_TILE_SAMPLING = os.environ.get("AIOSB_TILE_SAMPLING", "1") != "0"


# The CandidateGroup step writes the next forward's embedded rows itself (one
# kernel fewer per decode step); AIOSB_EMBED_IN_STEP=0 keeps the embedding kernel.
_EMBED_IN_STEP = os.environ.get("AIOSB_EMBED_IN_STEP", "1") != "0"


def _stat_trunk(model) -> bool:
    """Whether the model's decode forward is the standard-residual trunk of
    Qwen3Model.forward_stats (the one that takes pre-embedded rows)."""
    from ..attention import B200AttentionBackend
    from ..models.qwen3 import Qwen3ForCausalLM, Qwen3Model

    return (isinstance(model, Qwen3ForCausalLM) and type(model.model) is Qwen3Model
            and isinstance(model.attn_backend, B200AttentionBackend))


def stage_class(prefix_len: int) -> int:
    return next((c for c in STAGE_CLASSES if prefix_len <= c), STAGE_CLASSES[-1])


@dataclass
class RoundResult:
    output_ids: np.ndarray  # [attempts, max_new] int32 (pad where nothing was emitted)
    token_logprobs: np.ndarray  # [attempts, max_new] float32
    counts: list[int]
    logprob_sums: list[float]
    stop_codes: list[int]
    pages_consumed: int  # FIFO entries this round took (freed by the caller)
    active_model_tokens: int
    cancelled: bool
    steps: int


class CandidateGroupRuntime:
    def __init__(self, llm, max_rows: int = 16, max_steps: int = 64, max_banned: int = 64,
                 max_banned_width: int = 64) -> None:
        self.llm = llm
        dev = llm.device
        self.device = dev
        self.max_rows = max_rows
        self.max_steps = max_steps
        self.max_banned = max_banned
        self.max_banned_width = max_banned_width
        self.vocab = llm.config.vocab_size
        i32 = dict(dtype=torch.int32, device=dev)
        # The state and the round's results share one device block, so that the
        # round ends with one device-to-host copy (plus the status word):
        # [state | output_ids | token_logprobs | counts | logprob_sums | stop_codes]
        state_size = ctypes.sizeof(_lib.GroupState)
        state_words = (state_size + 7) // 8 * 2  # keeps every part 8-byte aligned
        rs = max_rows * max_steps
        self._out_offsets = offs = {}
        total = 0
        for name, words in (("state", state_words), ("ids", rs), ("lp", rs), ("counts", max_rows),
                            ("sums", max_rows), ("stops", max_rows)):
            offs[name] = total
            total += words
        self._out_dev = torch.zeros(total, **i32)
        self._out_host = torch.zeros(total, dtype=torch.int32).pin_memory()
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()

        def part(buf, name, words, dtype=torch.int32):
            return buf[offs[name] : offs[name] + words].view(dtype)

        self._out_part = part
        self.state = part(self._out_dev, "state", state_words).view(torch.uint8)[:state_size]
        self._state_host = torch.zeros(ctypes.sizeof(_lib.GroupState), dtype=torch.uint8).pin_memory()
        self._state_struct = _lib.GroupState.from_address(self._state_host.data_ptr())
        self.logits = torch.zeros((max_rows, self.vocab), dtype=torch.bfloat16, device=dev)
        self.uniforms = torch.zeros((max_rows, max_steps), dtype=torch.float32, device=dev)
        self.output_ids = part(self._out_dev, "ids", rs).view(max_rows, max_steps)
        self.token_logprobs = part(self._out_dev, "lp", rs, torch.float32).view(max_rows, max_steps)
        self.counts = part(self._out_dev, "counts", max_rows)
        self.logprob_sums = part(self._out_dev, "sums", max_rows, torch.float32)
        self.stop_codes = part(self._out_dev, "stops", max_rows)
        self.active = torch.zeros(max_rows, **i32)
        self.finished = torch.zeros(max_rows, **i32)
        self.tokens = torch.zeros(max_rows, **i32)
        self.positions = torch.zeros(max_rows, **i32)
        self.seq_lens = torch.zeros(max_rows, **i32)
        self.out_loc = torch.zeros(max_rows, **i32)
        self.row_page = torch.zeros(max_rows, **i32)
        self.row_table = torch.zeros(max_rows, **i32)
        # id lists in one device buffer, filled by one H2D copy per round:
        # [terminal ids | min-length ids | banned lengths | banned sequences]
        self._ids_host = torch.zeros(MAX_TERMINAL + MAX_MINLEN + max_banned * (1 + max_banned_width),
                                     dtype=torch.int32).pin_memory()
        self._ids_dev = torch.zeros_like(self._ids_host, device=dev)
        self._off_len = MAX_TERMINAL + MAX_MINLEN
        self._off_seq = self._off_len + max_banned
        self.cancel_flag = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.host_mirror = torch.zeros(4, dtype=torch.int32).pin_memory()
        self._mirror_np = self.host_mirror.numpy()
        self._done_event = torch.cuda.Event()
        state_i32 = self.state.view(torch.int32)
        self.prefix_len_view = state_i32[3:4]  # aiosb_group_state.prefix_len (offset 12)
        self.ptrs = _lib.GroupPtrs(
            state=self.state.data_ptr(),
            cancel_flag=ops.host_device_pointer(self.cancel_flag),
            host_mirror=ops.host_device_pointer(self.host_mirror),
            logits=self.logits.data_ptr(),
            uniforms=self.uniforms.data_ptr(),
            output_ids=self.output_ids.data_ptr(),
            token_logprobs=self.token_logprobs.data_ptr(),
            counts=self.counts.data_ptr(),
            logprob_sums=self.logprob_sums.data_ptr(),
            stop_codes=self.stop_codes.data_ptr(),
            active=self.active.data_ptr(),
            finished=self.finished.data_ptr(),
            tokens=self.tokens.data_ptr(),
            positions=self.positions.data_ptr(),
            seq_lens=self.seq_lens.data_ptr(),
            out_loc=self.out_loc.data_ptr(),
            row_page=self.row_page.data_ptr(),
            row_table=self.row_table.data_ptr(),
            terminal_ids=self._ids_dev.data_ptr(),
            minlen_ids=self._ids_dev[MAX_TERMINAL:].data_ptr(),
            banned=self._ids_dev[self._off_seq :].data_ptr(),
            banned_len=self._ids_dev[self._off_len :].data_ptr(),
            page_table=llm.ctx.page_table.data_ptr(),
            ring=llm.cache_manager.ring.data_ptr(),
            status=ops.status_word(dev).data_ptr(),
        )
        # The step also embeds the tokens it samples for the next forward when that
        # forward is the standard-residual trunk (it starts at its first linear)
        self.pre_embedded = None
        if _EMBED_IN_STEP and _stat_trunk(llm.model):
            hidden = llm.config.hidden_size
            emb_w = llm.model.model.embed_tokens.weight
            self._emb_out = torch.zeros((max_rows, hidden), dtype=emb_w.dtype, device=dev)
            self._emb_x = torch.zeros((max_rows, hidden), dtype=torch.float32, device=dev)
            self._emb_ss = torch.zeros((1, max_rows), dtype=torch.float32, device=dev)
            self.ptrs.embed_w = emb_w.data_ptr()
            self.ptrs.embed_out = self._emb_out.data_ptr()
            self.ptrs.embed_stat_x = self._emb_x.data_ptr()
            self.ptrs.embed_stat_ss = self._emb_ss.data_ptr()
            self.ptrs.hidden = hidden
            self.pre_embedded = (self._emb_out, self._emb_x, self._emb_ss)
        # [vocab / 16, rows, 4] tile statistics of the decode logits, and per row
        # count whether the LM head of that count's step graph writes them (known
        # after the graph's eager warm-up forward)
        self.tile_stats = (torch.zeros(self.vocab // 16 * max_rows * 4, dtype=torch.float32, device=dev)
                           if _TILE_SAMPLING and self.vocab % 16 == 0 else None)
        self._tile_rows: dict[int, bool] = {}
        # the steps inside a step graph follow that graph's forward
        # (GROUP_AFTER_FORWARD: the step reads its state while the LM head runs)
        self._ptrs_graph = _lib.GroupPtrs.from_buffer_copy(self.ptrs)
        self._ptrs_graph.flags = _lib.GROUP_AFTER_FORWARD
        self._ptrs_tiles = None
        if self.tile_stats is not None:
            self._ptrs_tiles = _lib.GroupPtrs.from_buffer_copy(self._ptrs_graph)
            self._ptrs_tiles.tile_stats = self.tile_stats.data_ptr()
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_launches: dict[int, int] = {}
        self.h2d_bytes = 0  # host->device bytes copied by rounds (bench accounting)
        self.d2h_bytes = 0
        self._pool = None
        # When `record` is set, every round's parameters and results are kept in
        # `rounds` (used by parity tests to replay the round on the CPU oracle).
        self.record = False
        self.rounds: list[tuple[dict, RoundResult]] = []
        # With `record_logits`, each round also keeps the logits every step sampled
        # from ([attempts, vocab] fp32 per step; synchronises after every step).
        self.record_logits = False
        self.step_logits: list[torch.Tensor] = []
        self._step_plan = self._persistent_plan() if _PERSISTENT else None
        self.history_mode = _HISTORY

    def use_history_mode(self, mode: str) -> None:
        """Selects the decode attention's history mode (a HISTORY_MODES name) for
        this runtime's step graphs; captured graphs are dropped."""
        self.history_mode = HISTORY_MODES[mode]
        self._tile_rows.clear()
        self._graphs.clear()
        self._graph_launches.clear()

    def use_persistent_step(self, enabled: bool = True) -> bool:
        """Switches this runtime's decode forward to (or away from) the persistent
        decode-step kernel; returns whether it is now in use (False when the model
        is not one the kernel serves). Captured step graphs are dropped."""
        self._step_plan = self._persistent_plan() if enabled else None
        self._tile_rows.clear()
        self._graphs.clear()
        self._graph_launches.clear()
        return self._step_plan is not None

    # ------------------------------------------------------- persistent step
    def _persistent_plan(self):
        """Device buffers and argument block of aiosb_decode_step, or None when
        the model is not one the persistent kernel serves."""
        from ..models.qwen3 import Qwen3ForCausalLM

        llm, cfg = self.llm, self.llm.config
        model = llm.model
        if (not isinstance(model, Qwen3ForCausalLM) or cfg.residual_type != "standard"
                or type(model.attn_backend).__name__ != "B200AttentionBackend"):
            return None  # the Block AttnRes trunk keeps the per-kernel forward
        if (cfg.hidden_size != 768 or cfg.intermediate_size != 2048 or cfg.head_dim not in (64, 96)
                or cfg.num_qo_heads % cfg.num_kv_heads or cfg.num_qo_heads // cfg.num_kv_heads > 7
                or cfg.num_qo_heads * cfg.head_dim != 768 or cfg.vocab_size % 16 or self.max_rows > 16):
            return None
        dev = self.device
        kv = llm.mha_kv_cache
        layers = model.model.layers.op_list
        descs = (_lib.DecodeLayer * len(layers))()
        for i, layer in enumerate(layers):
            at, mlp = layer.self_attn, layer.mlp
            descs[i] = _lib.DecodeLayer(
                w_qkv=at.qkv_proj.weight.data_ptr(), w_o=at.o_proj.weight.data_ptr(),
                w_gate_up=mlp.gate_up_proj.packed_weight().data_ptr(), w_down=mlp.down_proj.weight.data_ptr(),
                in_norm=layer.input_layernorm.weight.data_ptr(),
                post_norm=layer.post_attention_layernorm.weight.data_ptr(),
                q_norm=at.q_norm.weight.data_ptr(), k_norm=at.k_norm.weight.data_ptr(),
                k_cache=kv.k_slots(i).data_ptr(), v_cache=kv.v_slots(i).data_ptr(),
            )
        lib = _lib.load()
        work_bytes = int(lib.aiosb_decode_step_work_bytes(cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim))
        plan = dict(
            layers=torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).to(dev),
            # flagged activation lines passed between the kernel's phases (zero = no flag yet)
            work=torch.zeros(work_bytes // 4, dtype=torch.int32, device=dev),
            sync=torch.zeros(int(lib.aiosb_decode_step_sync_words()), dtype=torch.int32, device=dev),
        )
        cos, sin = model.model._rotary_emb.tables()
        embed = model.model.embed_tokens.weight
        plan["args"] = _lib.DecodeStepArgs(
            layers=plan["layers"].data_ptr(), num_layers=len(layers), rows=self.max_rows, hidden=768,
            intermediate=2048,
            num_qo_heads=cfg.num_qo_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
            vocab=cfg.vocab_size, eps=cfg.rms_norm_eps, scale=cfg.head_dim ** -0.5,
            embed=embed.data_ptr(), final_norm=model.model.norm.weight.data_ptr(),
            lm_head=model.lm_head._w().data_ptr(),
            tokens=self.tokens.data_ptr(), positions=self.positions.data_ptr(), out_loc=self.out_loc.data_ptr(),
            row_table=self.row_table.data_ptr(), seq_lens=self.seq_lens.data_ptr(),
            prefix_len=self.prefix_len_view.data_ptr(), active=self.active.data_ptr(),
            page_table=llm.ctx.page_table.data_ptr(), table_stride=llm.ctx.page_table.stride(0),
            num_slots=kv.num_slots, cos_tab=cos.data_ptr(), sin_tab=sin.data_ptr(), max_pos=cos.shape[0],
            work=plan["work"].data_ptr(), logits=self.logits.data_ptr(), logits_stride=self.logits.stride(0),
            sync=plan["sync"].data_ptr(), status=ops.status_word(dev).data_ptr(), wait_limit_ns=0,
            test_flag_skew=0, grid_ctas=0,
        )
        self._keep = (plan, descs)  # weights and buffers the argument block points to
        return plan

    def _decode_step(self, rows: int) -> None:
        args = _lib.DecodeStepArgs.from_buffer_copy(self._step_plan["args"])
        args.rows = rows
        _lib.call("aiosb_decode_step", ctypes.byref(args), self._stream())

    # ------------------------------------------------------------------ graphs
    def _decode_batch(self, rows: int, stage: int = STAGE_CLASSES[0]) -> Batch:
        reqs = [Req(input_ids=torch.empty(1, dtype=torch.long), cached_len=0, output_len=1, uid=i,
                    sampling_params=SamplingParams(max_tokens=1), table_idx=i) for i in range(rows)]
        batch = Batch(reqs=reqs, phase="decode", logits_out=self.logits[:rows], tile_stats_out=self.tile_stats)
        if self.pre_embedded is not None:
            out, x, ss = self.pre_embedded
            batch.pre_embedded = (out[:rows], ops.RowStats(x[:rows], ss[:, :rows]))
        batch.input_ids = self.tokens[:rows]
        batch.positions = self.positions[:rows]
        batch.out_loc = self.out_loc[:rows]
        batch.attn_metadata = B200AttentionMetadata(
            phase="decode", positions=self.positions[:rows], out_loc=self.out_loc[:rows],
            row_table=self.row_table[:rows], seq_lens=self.seq_lens[:rows], prefix_len=self.prefix_len_view,
            active=self.active[:rows], stable_history=self.history_mode, staged_prefix=stage,
        )
        return batch

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _group_step(self, rows: int, large: bool = False, after_forward: bool = False) -> None:
        # top_k_max: the largest sorted candidate set a round of this graph may ask for
        top_k_max = self.vocab if large else SORT_K
        if not after_forward:
            ptrs = self.ptrs  # a round's first step, after group_begin
        elif self._tile_rows.get(rows, False):
            ptrs = self._ptrs_tiles
        else:
            ptrs = self._ptrs_graph
        _lib.call("aiosb_group_step", ctypes.byref(ptrs), rows, self.vocab, top_k_max, self._stream())

    def _forward_and_step(self, rows: int, batch: Batch, large: bool = False) -> None:
        """One decode step after a round's first: the forward on the tokens the
        previous step sampled, then the step that samples its logits."""
        if self._step_plan is not None:
            self._decode_step(rows)
        else:
            with self.llm.ctx.forward_batch(batch):
                self.llm.model.forward()
        self._group_step(rows, large, after_forward=True)

    def _graph(self, rows: int, large: bool = False, stage: int = STAGE_CLASSES[0]) -> torch.cuda.CUDAGraph:
        """The step graph for `rows` rows; `large` steps sort whole rows (sorted
        candidate sets above SORT_K); `stage` is the prefix-length class the decode
        attention stages before its wait."""
        key = (rows, large, stage)
        graph = self._graphs.get(key)
        if graph is not None:
            return graph
        batch = self._decode_batch(rows, stage)
        # Eager warm-up with the group marked done: every kernel runs once (its
        # attributes get set) while all rows are inactive, so nothing is written.
        self._write_state(dict(done=1, rows=rows, max_steps=2, vocab=self.vocab, page_size=1, capacity=1,
                               table_stride=self.llm.ctx.page_table.stride(0)))
        self.active.zero_()
        self._forward_and_step(rows, batch, large)
        torch.cuda.synchronize(self.device)
        # the step kernel reads tile statistics only where this forward wrote them
        self._tile_rows[rows] = batch.tile_stats_written and self._step_plan is None
        graph = torch.cuda.CUDAGraph()
        before = _lib.launches
        with torch.cuda.graph(graph, pool=self._pool):
            self._forward_and_step(rows, batch, large)
        self._graph_launches[key] = _lib.launches - before
        _lib.launches = before
        if self._pool is None:
            self._pool = graph.pool()
        torch.cuda.synchronize(self.device)
        self._graphs[key] = graph
        return graph

    # ------------------------------------------------------------------ round
    def _write_state(self, fields: dict) -> None:
        ctypes.memset(self._state_host.data_ptr(), 0, ctypes.sizeof(_lib.GroupState))
        for name, value in fields.items():
            setattr(self._state_struct, name, value)
        self.state.copy_(self._state_host, non_blocking=True)

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
        terminal_ids: list[int],
        minlen_ids: list[int],
        banned_sequences: list[list[int]],
        ban_min_prefix: int,
        eos_id: int,
        pad_id: int,
        cancellation=None,
    ) -> RoundResult:
        if not 1 <= attempts <= self.max_rows:
            raise ValueError(f"attempts must be in [1, {self.max_rows}]")
        if max_new_tokens > self.max_steps:
            raise ValueError(f"max_new_tokens above the runtime's {self.max_steps}")
        if len(terminal_ids) > MAX_TERMINAL or len(minlen_ids) > MAX_MINLEN:
            raise ValueError("too many terminal / minimum-length ids")
        if len(banned_sequences) > self.max_banned or any(len(s) > self.max_banned_width for s in banned_sequences):
            raise ValueError("refill ban list exceeds the runtime's capacity")
        greedy = (temperature <= 0.0 or top_k == 1) and top_p == 1.0
        sort_k = min(top_k, self.vocab) if top_k > 0 else (self.vocab if top_p < 1.0 else 0)
        large = not greedy and sort_k > SORT_K
        if large and self.vocab > LARGE_SORT_VOCAB:
            raise ValueError(f"a sorted candidate set of {sort_k} needs a vocabulary of at most {LARGE_SORT_VOCAB}")
        cm = self.llm.cache_manager
        stage = stage_class(prefix_len)
        graph = self._graph(attempts, large, stage)
        head0 = cm.head
        width = max((len(s) for s in banned_sequences), default=0)
        self._write_state(dict(
            step=0, max_steps=max_new_tokens, min_new_tokens=min_new_tokens, prefix_len=prefix_len,
            row_offset=row_offset, rows=attempts, vocab=self.vocab, eos_id=eos_id, pad_id=pad_id,
            greedy=int(greedy), top_k=top_k, temperature=temperature, top_p=top_p, page_size=cm.page_size,
            n_terminal=len(terminal_ids), n_minlen=len(minlen_ids), n_banned=len(banned_sequences),
            banned_width=width, ban_min_prefix=ban_min_prefix, head=cm.head, tail=cm.tail,
            capacity=cm.num_pages, table_stride=self.llm.ctx.page_table.stride(0),
        ))
        ids = self._ids_host.numpy()
        ids[:MAX_TERMINAL + MAX_MINLEN] = 0
        ids[: len(terminal_ids)] = terminal_ids
        ids[MAX_TERMINAL : MAX_TERMINAL + len(minlen_ids)] = minlen_ids
        off_len, off_seq = self._off_len, self._off_seq
        for b, seq in enumerate(banned_sequences):
            ids[off_len + b] = len(seq)
            row = np.full(self.max_banned_width, pad_id, dtype=np.int32)
            row[: len(seq)] = seq
            ids[off_seq + b * width : off_seq + (b + 1) * width] = row[:width]
        n_ids = off_seq + len(banned_sequences) * width
        self._ids_dev[:n_ids].copy_(self._ids_host[:n_ids], non_blocking=True)
        self.cancel_flag.zero_()
        self._mirror_np[:] = 0
        if cancellation is not None:
            cancellation._attach_flag(self.cancel_flag)
        _lib.call("aiosb_group_begin", ctypes.byref(self.ptrs), prefix_logits.data_ptr(), seed & (2**64 - 1),
                  attempts, attempts, self._stream())
        self.h2d_bytes += self._state_host.numel() + 4 * n_ids
        launched = 0
        step_logits: list[torch.Tensor] = []
        if self.record_logits:
            torch.cuda.synchronize(self.device)
            step_logits.append(prefix_logits.float().cpu().expand(attempts, -1).clone())
        for step in range(max_new_tokens):
            if cancellation is not None and cancellation.cancelled:
                break
            if step >= 2:
                # keep <= 2 steps queued; stop once the device reports completion
                while int(self._mirror_np[0]) < step - 1 and not int(self._mirror_np[1]):
                    time.sleep(0)
                if int(self._mirror_np[1]):
                    break
            if step == 0:
                self._group_step(attempts, large)  # samples the broadcast prefix row
            else:
                graph.replay()  # the forward on step - 1's tokens, then step `step`
                _lib.count_launches(self._graph_launches[(attempts, large, stage)])
                if self.record_logits:
                    torch.cuda.synchronize(self.device)
                    step_logits.append(self.logits[:attempts].float().cpu())
            launched += 1
        # [rows, steps] arrays use the round's max_new_tokens as their row stride
        n = attempts * max_new_tokens
        # one copy of the result block and one of the status word: the status is
        # checked from the host copy, without a second synchronising read
        self._out_host.copy_(self._out_dev, non_blocking=True)
        self._status_host.copy_(ops.status_word(self.device), non_blocking=True)
        self.d2h_bytes += 4 * (self._out_host.numel() + 1)
        self._done_event.record()
        self._done_event.synchronize()
        if cancellation is not None:
            cancellation._detach_flag(self.cancel_flag)
        if int(self._status_host[0]) != 0:
            ops.check_status(self.device)  # raises, and resets the word
        host = self._out_host
        part = self._out_part
        state_words = self._out_offsets["ids"]
        final = _lib.GroupState.from_buffer_copy(part(host, "state", state_words).numpy().tobytes())
        res_ids = part(host, "ids", n).numpy()
        res_lp = part(host, "lp", n, torch.float32).numpy()
        consumed = int(final.head) - head0
        cm.advance_head(int(final.head))
        host_cancelled = cancellation is not None and cancellation.cancelled and launched < max_new_tokens
        result = RoundResult(
            output_ids=res_ids.reshape(attempts, max_new_tokens).copy(),
            token_logprobs=res_lp.reshape(attempts, max_new_tokens).copy(),
            counts=part(host, "counts", attempts).tolist(),
            logprob_sums=part(host, "sums", attempts, torch.float32).tolist(),
            stop_codes=part(host, "stops", attempts).tolist(),
            pages_consumed=consumed,
            active_model_tokens=int(final.active_model_tokens),
            cancelled=bool(final.cancelled) or host_cancelled,
            steps=int(final.step),
        )
        if self.record:
            self.rounds.append((dict(
                prefix_len=prefix_len, row_offset=row_offset, attempts=attempts, max_new_tokens=max_new_tokens,
                min_new_tokens=min_new_tokens, seed=seed, temperature=temperature, top_k=top_k, top_p=top_p,
                banned_sequences=[list(x) for x in banned_sequences], ban_min_prefix=ban_min_prefix,
                head=head0, step_logits=step_logits,
            ), result))
        return result
