"""Prefix prefill of one request (the keystroke prefix) as replayed CUDA graphs.

A keystroke prefills its whole prefix, or only the tokens past the reused
token-LCP (aios/ime.py:1170-1217). Every input of that forward — new token ids,
positions, KV slots, the attention request/tile arrays and the full prefix slot
list — travels in one host-to-device copy into a fixed device buffer, and the
forward itself (every layer's kernels, the LM head on the last token) replays as
a CUDA graph captured once per new-token count. A page-table reset kernel writes
the prefix slots into every candidate row. Counts above ``MAX_GRAPH_TOKENS`` run
the same kernels without a graph.
"""

from __future__ import annotations

import torch

from .. import _lib
from ..attention import B200AttentionMetadata
from ..core import Batch, Req, SamplingParams
from ..kernel import ops


class PrefixRunner:
    MAX_GRAPH_TOKENS = 64

    def __init__(self, llm) -> None:
        self.llm = llm
        dev = llm.device
        self.device = dev
        self.max_pos = llm.config.max_position_embeddings
        self.tile_tokens = llm.model.attn_backend.tile_tokens
        self.max_tiles = -(-self.max_pos // self.tile_tokens)
        mp = self.max_pos
        self.off_ids, self.off_pos, self.off_loc = 0, mp, 2 * mp
        self.off_meta = 3 * mp
        self.off_slots = self.off_meta + 4 + 2 * self.max_tiles
        total = self.off_slots + mp
        self._host = torch.zeros(total, dtype=torch.int32).pin_memory()
        self._host_np = self._host.numpy()
        self._dev = torch.zeros(total, dtype=torch.int32, device=dev)
        self._copied = torch.cuda.Event()
        self._pending = False
        self.logits = torch.zeros((1, llm.config.vocab_size), dtype=torch.bfloat16, device=dev)
        self._graphs: dict[int, tuple[torch.cuda.CUDAGraph, int]] = {}
        self._pool = None
        self.h2d_bytes = 0

    @property
    def slots_dev(self) -> torch.Tensor:
        return self._dev[self.off_slots :]

    def _batch(self, n: int) -> Batch:
        req = Req(input_ids=torch.empty(n, dtype=torch.long), cached_len=0, output_len=1, uid=0,
                  sampling_params=SamplingParams(max_tokens=1), table_idx=0)
        batch = Batch(reqs=[req], phase="prefill", logits_out=self.logits)
        d = self._dev
        batch.input_ids = d[self.off_ids : self.off_ids + n]
        batch.positions = d[self.off_pos : self.off_pos + n]
        batch.out_loc = d[self.off_loc : self.off_loc + n]
        tiles = -(-n // self.tile_tokens)
        batch.attn_metadata = B200AttentionMetadata(
            phase="prefill", positions=batch.positions, out_loc=batch.out_loc, last_rows=(n - 1,),
            meta=d[self.off_meta : self.off_meta + 4 + 2 * tiles], num_requests=1, num_tiles=tiles,
            tile_tokens=self.tile_tokens, max_q_len=n,
        )
        return batch

    def fill_table(self, table: torch.Tensor, rows: int, width: int, n: int) -> None:
        _lib.call("aiosb_page_table_fill", table.data_ptr(), table.stride(0), rows, width,
                  self.slots_dev.data_ptr(), n, torch.cuda.current_stream(self.device).cuda_stream)

    def run(self, token_ids: list[int], cached_len: int, slots: list[int], table: torch.Tensor, rows: int,
            width: int) -> torch.Tensor:
        """Prefill tokens [cached_len, len) whose KV goes to slots[cached_len:];
        resets `rows` page-table rows to the prefix; returns the [1, V] logits of
        the last token (a buffer the next prefill overwrites)."""
        T = len(token_ids)
        n = T - cached_len
        if n < 1:
            raise ValueError("prefill needs at least one new token")
        if self._pending:
            self._copied.synchronize()  # the staging buffer is still being read
        h = self._host_np
        tiles = -(-n // self.tile_tokens)
        h[self.off_ids : self.off_ids + n] = token_ids[cached_len:]
        h[self.off_pos : self.off_pos + n] = range(cached_len, T)
        h[self.off_loc : self.off_loc + n] = slots[cached_len:]
        meta = [0, n, cached_len, 0, *([0] * tiles), *range(0, n, self.tile_tokens)]
        h[self.off_meta : self.off_meta + len(meta)] = meta
        h[self.off_slots : self.off_slots + T] = slots
        end = self.off_slots + T
        self._dev[:end].copy_(self._host[:end], non_blocking=True)
        self._copied.record()
        self._pending = True
        self.h2d_bytes += 4 * end
        self.fill_table(table, rows, width, T)
        entry = self._graphs.get(n)
        if entry is not None:
            entry[0].replay()
            _lib.count_launches(entry[1])
            return self.logits
        batch = self._batch(n)
        with self.llm.ctx.forward_batch(batch):
            self.llm.model.forward()
        if n <= self.MAX_GRAPH_TOKENS:
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            before = _lib.launches
            with torch.cuda.graph(graph, pool=self._pool):
                with self.llm.ctx.forward_batch(batch):
                    self.llm.model.forward()
            launches = _lib.launches - before
            _lib.launches = before
            if self._pool is None:
                self._pool = graph.pool()
            self._graphs[n] = (graph, launches)
        return self.logits
