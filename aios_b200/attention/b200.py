"""B200 attention backend: the plugin that replaces FlashInferAttentionBackend
(aios/attention/flashinfer.py:115-394).

Prefill runs the sm_100a prologue kernel (q/k RMSNorm + bf16 RoPE + KV store) and
the causal paged prefill kernel; decode runs the cascade decode kernel, which
reads each shared-prefix KV slot once per KV head for all candidate rows. The
reference slot API ``forward(q, k, v, ...)`` (already normalised and rotated q/k)
is served by the KV-store kernel plus the same attention kernels.

Metadata is device-resident: ``prepare_metadata`` uploads the few per-request
integers once per batch (no host-side planning step), and the CandidateGroup
runtime builds a static decode metadata object whose tensors its step kernel
rewrites on the device, so decode steps replay as CUDA graphs.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING

import torch

from ..core import get_global_ctx
from ..kernel import ops
from .base import BaseAttentionBackend, BaseAttentionMetadata

if TYPE_CHECKING:
    from ..core import Batch
    from ..kvcache import MHAKVCache
    from ..models.config import ModelConfig

SUPPORTED_HEAD_DIMS = frozenset({64, 96, 128})


@dataclass
class B200AttentionMetadata(BaseAttentionMetadata):
    phase: str
    positions: torch.Tensor  # int32 [tokens]
    out_loc: torch.Tensor  # int32 [tokens]
    cu_seqlens_q: torch.Tensor | None = None  # int32 [bs + 1] (prefill)
    last_rows: tuple[int, ...] = ()
    meta: torch.Tensor | None = None  # int32 request + tile arrays (prefill)
    num_requests: int = 0
    num_tiles: int = 0
    tile_tokens: int = 0
    max_q_len: int = 0  # longest request of a prefill batch (new tokens); 0 = unknown
    row_table: torch.Tensor | None = None  # int32 [rows] (decode)
    seq_lens: torch.Tensor | None = None  # int32 [rows] (decode)
    prefix_len: torch.Tensor | None = None  # int32 [1]: shared prefix keys (decode)
    active: torch.Tensor | None = None  # int32 [rows] (decode)
    # decode: the row table, prefix length and every key before the current
    # position were written by earlier launches (the CandidateGroup runtime)
    stable_history: bool | int = False  # aiosb_attention_decode's history mode (0, 1 staged, 2 prefix-once)
    staged_prefix: int = 0  # bound on the prefix keys staged before the wait (0: the kernel's default)

    def get_last_indices(self, bs: int) -> torch.Tensor:
        assert self.cu_seqlens_q is not None, "last indices exist for prefill batches"
        return self.cu_seqlens_q[1 : 1 + bs].to(torch.long) - 1


def _to_device_i32(values: list[int], device: torch.device) -> torch.Tensor:
    host = torch.tensor(values, dtype=torch.int32).pin_memory()
    ops.transfer_bytes["h2d"] += 4 * len(values)
    return host.to(device, non_blocking=True)


class B200AttentionBackend(BaseAttentionBackend):
    def __init__(self, config: ModelConfig, workspace_size: int = 0) -> None:
        if config.head_dim not in SUPPORTED_HEAD_DIMS:
            raise ValueError(f"head_dim {config.head_dim} unsupported (64, 96, 128)")
        if config.num_qo_heads % config.num_kv_heads:
            raise ValueError("query head count must be divisible by KV head count")
        self.num_heads = config.num_qo_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self.sm_scale = config.head_dim**-0.5
        self.eps = config.rms_norm_eps
        self.backend_name = "b200-cascade"
        self.workspace_size = workspace_size  # accepted for API parity; no workspace is used
        self.tile_tokens = ops.prefill_tile_tokens(self.num_heads, self.num_kv_heads)

    # -- metadata --------------------------------------------------------------
    def prepare_metadata(self, batch: Batch) -> B200AttentionMetadata:
        ctx = get_global_ctx()
        device = ctx.page_table.device
        positions = batch.positions.to(device=device, dtype=torch.int32)
        out_loc = batch.out_loc.to(device=device, dtype=torch.int32).view(-1)
        reqs = batch.reqs
        if batch.is_prefill:
            q_lens = [r.extend_len for r in reqs]
            cu = [0]
            for n in q_lens:
                cu.append(cu[-1] + n)
            meta_host, num_tiles = ops.prefill_meta(
                q_lens, [r.cached_len for r in reqs], [int(r.table_idx) for r in reqs], self.tile_tokens
            )
            md = B200AttentionMetadata(
                phase="prefill",
                positions=positions,
                out_loc=out_loc,
                cu_seqlens_q=_to_device_i32(cu, device),
                last_rows=tuple(c - 1 for c in cu[1:]),
                meta=_to_device_i32(meta_host, device),
                num_requests=len(reqs),
                num_tiles=num_tiles,
                tile_tokens=self.tile_tokens,
                max_q_len=max(q_lens, default=0),
            )
        else:
            packed = _to_device_i32([int(r.table_idx) for r in reqs] + [r.device_len for r in reqs], device)
            md = B200AttentionMetadata(
                phase="decode",
                positions=positions,
                out_loc=out_loc,
                row_table=packed[: len(reqs)],
                seq_lens=packed[len(reqs) :],
            )
        batch.attn_metadata = md
        return md

    # -- fused path (raw qkv projection in) -------------------------------------
    def forward_qkv(
        self,
        qkv: torch.Tensor,
        q_norm_w: torch.Tensor,
        k_norm_w: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        paged_kv_cache: MHAKVCache,
        layer_id: int,
        batch: Batch,
    ) -> torch.Tensor:
        md = batch.attn_metadata
        assert isinstance(md, B200AttentionMetadata)
        ctx = get_global_ctx()
        tokens = qkv.shape[0]
        out = torch.empty((tokens, self.num_heads * self.head_dim), dtype=qkv.dtype, device=qkv.device)
        kc, vc = paged_kv_cache.k_slots(layer_id), paged_kv_cache.v_slots(layer_id)
        if md.phase == "prefill" and 1 <= md.max_q_len <= ops.FUSED_PREFILL_MAX_TOKENS:
            # short requests (a keystroke's prefix): norm, RoPE, K/V store and
            # attention in one launch; every cached key came from an earlier forward
            return ops.attention_prefill_fused(
                qkv=qkv, out=out, q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=self.eps, cos=cos, sin=sin,
                positions=md.positions, out_loc=md.out_loc, k_cache=kc, v_cache=vc, page_table=ctx.page_table,
                meta=md.meta, num_requests=md.num_requests, num_tiles=md.num_tiles, tile_tokens=md.tile_tokens,
                max_q_len=md.max_q_len, num_qo_heads=self.num_heads, num_kv_heads=self.num_kv_heads,
                head_dim=self.head_dim, scale=self.sm_scale,
            )
        if md.phase == "prefill":
            qbuf = torch.empty_like(out)
            ops.qk_norm_rope_store(
                qkv=qkv, num_qo_heads=self.num_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=self.eps, cos=cos, sin=sin, positions=md.positions,
                out_loc=md.out_loc, k_cache=kc, v_cache=vc, q_out=qbuf,
            )
            return self._prefill(qbuf, out, kc, vc, ctx.page_table, md)
        return ops.attention_decode(
            out=out, k_cache=kc, v_cache=vc, page_table=ctx.page_table, row_table=md.row_table,
            seq_lens=md.seq_lens, positions=md.positions, num_qo_heads=self.num_heads,
            num_kv_heads=self.num_kv_heads, head_dim=self.head_dim, scale=self.sm_scale, qkv=qkv,
            q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=self.eps, cos=cos, sin=sin, out_loc=md.out_loc,
            prefix_len=md.prefix_len, active=md.active, stable_history=md.stable_history,
            staged_prefix=md.staged_prefix,
        )

    # -- reference slot API (q/k already normalised and rotated) ---------------
    def forward(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        paged_kv_cache: MHAKVCache,
        layer_id: int,
        batch: Batch,
    ) -> torch.Tensor:
        md = batch.attn_metadata
        assert isinstance(md, B200AttentionMetadata)
        ctx = get_global_ctx()
        paged_kv_cache.store_kv(k, v, md.out_loc, layer_id)
        tokens = q.shape[0]
        q2 = q.reshape(tokens, self.num_heads * self.head_dim).contiguous()
        out = torch.empty_like(q2)
        kc, vc = paged_kv_cache.k_slots(layer_id), paged_kv_cache.v_slots(layer_id)
        if md.phase == "prefill":
            return self._prefill(q2, out, kc, vc, ctx.page_table, md)
        return ops.attention_decode(
            out=out, k_cache=kc, v_cache=vc, page_table=ctx.page_table, row_table=md.row_table,
            seq_lens=md.seq_lens, positions=md.positions, num_qo_heads=self.num_heads,
            num_kv_heads=self.num_kv_heads, head_dim=self.head_dim, scale=self.sm_scale, q=q2,
            prefix_len=md.prefix_len, active=md.active,
        )

    def _prefill(self, q, out, kc, vc, page_table, md: B200AttentionMetadata) -> torch.Tensor:
        return ops.attention_prefill(
            q=q, out=out, k_cache=kc, v_cache=vc, page_table=page_table, meta=md.meta,
            num_requests=md.num_requests, num_tiles=md.num_tiles, tile_tokens=md.tile_tokens,
            num_qo_heads=self.num_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
            scale=self.sm_scale,
        )
