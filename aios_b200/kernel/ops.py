"""Torch-tensor wrappers over the C ABI (``aios_b200._lib``).

Each wrapper validates shapes/dtypes on the host, passes raw device addresses and
the current CUDA stream, and never computes anything itself: every op here runs
as a hand-written sm_100a kernel. Device-side errors land in a per-device int32
status word that :func:`check_status` turns into a ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

_STATUS: dict[int, torch.Tensor] = {}

# Bytes the host side stages to / from the device outside the runtime's own
# counters (prefill ids, attention metadata); read by the benchmark.
transfer_bytes = {"h2d": 0, "d2h": 0}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32 status word that kernels report device faults into."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(index)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _STATUS[index] = st
    return st


def check_status(device: torch.device, reset: bool = True) -> None:
    """Raises if any kernel on `device` reported a device-side fault (syncs)."""
    st = status_word(device)
    code = int(st.item())
    if code:
        if reset:
            st.zero_()
        raise RuntimeError(f"aios_b200 device status {code}: {_lib.DEVICE_STATUS_NAMES.get(code, 'unknown')}")


def host_device_pointer(pinned: torch.Tensor) -> int:
    """Device address of a page-locked host tensor (for host-mapped flags)."""
    if not pinned.is_pinned():
        raise ValueError("host_device_pointer needs a pinned CPU tensor")
    out = ctypes.c_void_p()
    _lib.call("aiosb_host_device_pointer", pinned.data_ptr(), ctypes.byref(out))
    return int(out.value)


def _require_cuda(*tensors: torch.Tensor, what: str) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what} requires CUDA tensors")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# KV store (aios/kernel/store.py:32-61)
# ---------------------------------------------------------------------------
def store_cache(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    indices: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
) -> None:
    """Scatter a flat batch of K/V vectors into a contiguous CUDA cache."""
    if k_cache.ndim != 3 or v_cache.ndim != 3:
        raise ValueError("KV cache must have shape (num_slots, num_heads, head_dim)")
    if k.shape[1:] != k_cache.shape[1:] or v.shape[1:] != v_cache.shape[1:]:
        raise ValueError("K/V input shape does not match the cache layout")
    if indices.numel() != k.shape[0] or k.shape != v.shape:
        raise ValueError("KV write indices and K/V tensors must have matching token counts")
    _require_cuda(k_cache, v_cache, indices, k, v, what="store_cache")
    if k.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("store_cache expects bf16 K/V and cache")
    for name, t in (("k", k), ("v", v)):
        if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
            raise ValueError(f"{name} rows must be contiguous within a token")
    if not (k_cache[0].is_contiguous() and v_cache[0].is_contiguous()):
        raise ValueError("KV cache rows must be contiguous")
    idx = indices.to(torch.int32).contiguous()
    width = k_cache.shape[1] * k_cache.shape[2]
    _lib.call(
        "aiosb_kv_store",
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        k_cache.stride(0),
        k_cache.shape[0],
        idx.data_ptr(),
        k.shape[0],
        k.data_ptr(),
        k.stride(0),
        v.data_ptr(),
        v.stride(0),
        width,
        status_word(k.device).data_ptr(),
        _stream(k.device),
    )


# ---------------------------------------------------------------------------
# AttnRes mixer (aios/kernel/attnres.py:130-223)
# ---------------------------------------------------------------------------
def b200_attnres_mix(
    bank: torch.Tensor,
    partial: torch.Tensor | None,
    weighted_query: torch.Tensor,
    eps: float,
    *,
    score_buffer: torch.Tensor | None = None,
    output_buffer: torch.Tensor | None = None,
) -> torch.Tensor:
    """FP32 depth routing and BF16 value aggregation in one sm_100a kernel.

    Same signature and layout checks as the reference ``triton_attnres_mix``;
    ``score_buffer`` is accepted and validated but unused, because the fused
    kernel keeps the [S, N] scores in registers.
    """
    if not bank.is_cuda:
        raise ValueError("B200 AttnRes requires CUDA tensors")
    if bank.ndim != 3:
        raise ValueError("bank must have shape [S,N,D]")
    if not bank.is_contiguous():
        raise ValueError("bank must be contiguous for the B200 pointer layout")
    bank_sources, num_tokens, hidden_size = bank.shape
    if bank_sources < 1 or num_tokens < 1 or hidden_size < 1:
        raise ValueError("bank dimensions must be positive")
    total_sources = bank_sources + int(partial is not None)
    if partial is not None and partial.shape != bank.shape[1:]:
        raise ValueError("partial must match bank [N,D]")
    if partial is not None and not partial.is_contiguous():
        raise ValueError("partial must be contiguous")
    if weighted_query.shape != (hidden_size,):
        raise ValueError("weighted_query must match hidden size")
    if not weighted_query.is_contiguous():
        raise ValueError("weighted_query must be contiguous")
    if weighted_query.dtype != torch.float32:
        raise ValueError("weighted_query must be float32")
    if bank.dtype != torch.bfloat16 or (partial is not None and partial.dtype != torch.bfloat16):
        raise ValueError("B200 AttnRes expects bf16 bank/partial")
    if score_buffer is not None:
        if score_buffer.dtype != torch.float32 or score_buffer.device != bank.device:
            raise ValueError("score_buffer must be CUDA float32 on bank device")
        if (
            score_buffer.shape[0] < total_sources
            or score_buffer.shape[1] != num_tokens
            or not score_buffer.is_contiguous()
        ):
            raise ValueError("score_buffer must be contiguous [capacity_sources, num_tokens]")
    if output_buffer is None:
        output = torch.empty_like(bank[0])
    else:
        if output_buffer.shape != bank.shape[1:]:
            raise ValueError("output_buffer must match bank [N,D]")
        if output_buffer.dtype != bank.dtype or output_buffer.device != bank.device:
            raise ValueError("output_buffer must match bank dtype/device")
        if not output_buffer.is_contiguous():
            raise ValueError("output_buffer must be contiguous")
        output = output_buffer
    _lib.call(
        "aiosb_attnres_mix",
        bank.data_ptr(),
        bank_sources,
        num_tokens,
        hidden_size,
        _ptr(partial),
        weighted_query.data_ptr(),
        float(eps),
        output.data_ptr(),
        status_word(bank.device).data_ptr(),
        _stream(bank.device),
    )
    return output


def b200_attnres_mix_rmsnorm(
    bank: torch.Tensor,
    partial: torch.Tensor | None,
    weighted_query: torch.Tensor,
    eps: float,
    norm_weight: torch.Tensor,
    norm_eps: float,
    *,
    output_buffer: torch.Tensor | None = None,
    stable_sources: int = 0,
) -> torch.Tensor:
    """rmsnorm(b200_attnres_mix(bank, partial, weighted_query, eps)) * norm_weight
    in one kernel: the mixer and the RMSNorm that consumes its output in the Block
    AttnRes layers. The mixer result itself is not returned. ``stable_sources``:
    the first bank sources were written before the previous kernel on the stream
    began, so the kernel may read them before waiting on it."""
    if not (bank.is_cuda and bank.dtype == torch.bfloat16 and bank.ndim == 3 and bank.is_contiguous()):
        raise ValueError("bank must be a contiguous CUDA bf16 [S,N,D] tensor")
    sources, tokens, hidden = bank.shape
    if partial is not None and (partial.shape != bank.shape[1:] or not partial.is_contiguous()
                                or partial.dtype != torch.bfloat16):
        raise ValueError("partial must be a contiguous bf16 [N,D] tensor matching bank")
    if weighted_query.shape != (hidden,) or weighted_query.dtype != torch.float32:
        raise ValueError("weighted_query must be float32 [D]")
    if norm_weight.shape != (hidden,) or norm_weight.dtype != torch.bfloat16 or not norm_weight.is_contiguous():
        raise ValueError("norm_weight must be a contiguous bf16 [D] tensor")
    output = torch.empty_like(bank[0]) if output_buffer is None else output_buffer
    if output.shape != bank.shape[1:] or not output.is_contiguous():
        raise ValueError("output_buffer must be a contiguous [N,D] tensor")
    _lib.call(
        "aiosb_attnres_mix_rmsnorm",
        bank.data_ptr(), sources, tokens, hidden, _ptr(partial), weighted_query.contiguous().data_ptr(), float(eps),
        norm_weight.data_ptr(), float(norm_eps), int(stable_sources), output.data_ptr(), _stream(bank.device),
    )
    return output


MIX_MAX_SOURCES = 10  # aiosb_linear_attnres_rmsnorm: bank + partial
MIX_MAX_ROWS = 8


def linear_attnres_rmsnorm_eligible(bank: torch.Tensor, partial: torch.Tensor | None, stable: int) -> bool:
    sources, tokens, hidden = bank.shape
    late = sources - stable + (partial is not None)
    return (tokens <= MIX_MAX_ROWS and hidden == 768 and 0 <= stable <= sources and late <= 2
            and sources + (partial is not None) <= MIX_MAX_SOURCES)


def linear_attnres_rmsnorm(
    bank: torch.Tensor,
    partial: torch.Tensor | None,
    stable_sources: int,
    weighted_query: torch.Tensor,
    mix_eps: float,
    norm_weight: torch.Tensor,
    norm_eps: float,
    weight: torch.Tensor,
    *,
    epilogue: int = _lib.EPI_STORE,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``linear(rmsnorm(attnres_mix(bank, partial)) * norm_weight, weight)`` in one
    decode kernel (at most 8 tokens, hidden 768): the mixer's rows are built inside
    the linear. The first ``stable_sources`` bank sources were written before the
    previous kernel on the stream began."""
    if not linear_attnres_rmsnorm_eligible(bank, partial, stable_sources):
        raise ValueError("linear_attnres_rmsnorm: 1..8 tokens, hidden 768, <= 10 sources, <= 2 read late")
    _require_cuda(bank, weighted_query, norm_weight, weight, what="linear_attnres_rmsnorm")
    sources, tokens, hidden = bank.shape
    n = weight.shape[0]
    cols = n // 2 if epilogue == _lib.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((tokens, cols), dtype=bank.dtype, device=bank.device)
    _lib.call(
        "aiosb_linear_attnres_rmsnorm", bank.data_ptr(), sources, int(stable_sources), tokens, _ptr(partial),
        weighted_query.contiguous().data_ptr(), float(mix_eps), norm_weight.data_ptr(), float(norm_eps),
        weight.data_ptr(), n, hidden, out.data_ptr(), out.stride(0), epilogue, status_word(bank.device).data_ptr(),
        _stream(bank.device),
    )
    return out


# ---------------------------------------------------------------------------
# Norms / activations / embedding (aios/layers/{norm,activation,embedding}.py)
# ---------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dim of a 2-D [T, H] or 3-D [T, heads, d] view."""
    _require_cuda(x, weight, what="rmsnorm")
    if out is None:
        out = torch.empty_like(x)
    if x.ndim == 2:
        x3, o3 = x.unsqueeze(1), out.unsqueeze(1)
    elif x.ndim == 3:
        x3, o3 = x, out
    else:
        raise ValueError("rmsnorm expects a 2-D or 3-D tensor")
    hidden = x3.shape[2]
    if weight.shape != (hidden,):
        raise ValueError("rmsnorm weight must match the last dimension")
    for t in (x3, o3):
        if t.stride(2) != 1 or (t.shape[1] > 1 and t.stride(1) != hidden):
            raise ValueError("rmsnorm rows must be dense within a token")
    _lib.call(
        "aiosb_rmsnorm",
        x3.data_ptr(),
        x3.shape[0] * x3.shape[1],
        hidden,
        x3.shape[1],
        x3.stride(0),
        weight.data_ptr(),
        float(eps),
        o3.data_ptr(),
        o3.stride(0),
        _stream(x.device),
    )
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    """residual += x; x = rmsnorm(residual) (in place, FlashInfer semantics)."""
    _require_cuda(x, residual, weight, what="fused_add_rmsnorm")
    if x.shape != residual.shape or x.ndim != 2 or not x.is_contiguous() or not residual.is_contiguous():
        raise ValueError("fused_add_rmsnorm expects matching contiguous [T, H] tensors")
    _lib.call(
        "aiosb_add_rmsnorm",
        x.data_ptr(),
        residual.data_ptr(),
        x.shape[0],
        x.shape[1],
        weight.data_ptr(),
        float(eps),
        _stream(x.device),
    )


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(x, what="silu_and_mul")
    if x.ndim != 2 or x.shape[1] % 2 or not x.is_contiguous():
        raise ValueError("silu_and_mul expects a contiguous [T, 2F] tensor")
    f = x.shape[1] // 2
    if out is None:
        out = torch.empty((x.shape[0], f), dtype=x.dtype, device=x.device)
    _lib.call("aiosb_silu_mul", x.data_ptr(), x.shape[0], f, out.data_ptr(), _stream(x.device))
    return out


def embedding(ids: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(ids, weight, what="embedding")
    ids = ids.contiguous()
    if ids.dtype not in (torch.int64, torch.int32):
        raise ValueError("embedding ids must be int32 or int64")
    if out is None:
        out = torch.empty((ids.numel(), weight.shape[1]), dtype=weight.dtype, device=weight.device)
    _lib.call(
        "aiosb_embedding",
        ids.data_ptr(),
        int(ids.dtype == torch.int64),
        ids.numel(),
        weight.data_ptr(),
        weight.shape[0],
        weight.shape[1],
        out.data_ptr(),
        status_word(ids.device).data_ptr(),
        _stream(ids.device),
    )
    return out


# ---------------------------------------------------------------------------
# Linear (tcgen05 GEMM)
# ---------------------------------------------------------------------------
def linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    out: torch.Tensor | None = None,
    epilogue: int = _lib.EPI_STORE,
    residual: torch.Tensor | None = None,
    tile_stats: torch.Tensor | None = None,
    early_dependents: bool = False,
) -> torch.Tensor:
    """y = x @ weight.T on the tensor cores (bf16 in, fp32 accumulate, bf16 out).

    ``epilogue=EPI_ADD`` returns ``residual + bf16(x @ weight.T)`` (residual may
    be ``out`` for an in-place add). ``tile_stats`` and ``early_dependents`` as in
    ``linear_stat_norm``."""
    _require_cuda(x, weight, what="linear")
    if x.ndim != 2 or weight.ndim != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError("linear expects x [T, K] and weight [N, K]")
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("linear expects contiguous x and weight")
    n = weight.shape[0]
    cols = n // 2 if epilogue == _lib.EPI_SILU_MUL else n
    if epilogue == _lib.EPI_ADD:
        if residual is None or residual.shape != (x.shape[0], n) or residual.stride(1) != 1:
            raise ValueError("the add epilogue needs a residual [rows, n] with contiguous rows")
    if out is None:
        out = torch.empty((x.shape[0], cols), dtype=x.dtype, device=x.device)
    if out.stride(1) != 1:
        raise ValueError("linear output rows must be contiguous")
    if tile_stats is not None:
        _check_tile_stats(tile_stats, epilogue, x.shape[0], x.shape[1], n)
        _lib.call("aiosb_linear_tiles", x.data_ptr(), x.shape[0], x.shape[1], weight.data_ptr(), n, out.data_ptr(),
                  out.stride(0), tile_stats.data_ptr(), status_word(x.device).data_ptr(), _stream(x.device))
        return out
    _lib.call(
        "aiosb_linear",
        x.data_ptr(),
        x.shape[0],
        x.shape[1],
        weight.data_ptr(),
        n,
        out.data_ptr(),
        out.stride(0),
        epilogue | (_lib.LINEAR_EARLY_DEPENDENTS if early_dependents else 0),
        _ptr(residual) if epilogue == _lib.EPI_ADD else None,
        residual.stride(0) if (epilogue == _lib.EPI_ADD and residual is not None) else 0,
        status_word(x.device).data_ptr(),
        _stream(x.device),
    )
    return out


MAX_NORM_ROWS = 64  # rows the fused-RMSNorm GEMM prologue handles


def linear_rmsnorm(
    x: torch.Tensor,
    residual_in: torch.Tensor | None,
    norm_weight: torch.Tensor,
    eps: float,
    weight: torch.Tensor,
    *,
    residual_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    epilogue: int = _lib.EPI_STORE,
) -> torch.Tensor:
    """``linear(rmsnorm(x + residual_in) * norm_weight, weight)`` in one kernel
    (rows <= 64); ``residual_out`` receives ``x + residual_in`` when given."""
    _require_cuda(x, norm_weight, weight, what="linear_rmsnorm")
    rows, k = x.shape
    if rows > MAX_NORM_ROWS:
        raise ValueError(f"linear_rmsnorm handles at most {MAX_NORM_ROWS} rows")
    for t in (x, residual_in, residual_out):
        if t is not None and (t.shape != (rows, k) or not t.is_contiguous()):
            raise ValueError("linear_rmsnorm expects contiguous [rows, k] x / residual tensors")
    n = weight.shape[0]
    cols = n // 2 if epilogue == _lib.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((rows, cols), dtype=x.dtype, device=x.device)
    _lib.call(
        "aiosb_linear_rmsnorm",
        x.data_ptr(),
        _ptr(residual_in),
        _ptr(residual_out),
        norm_weight.data_ptr(),
        float(eps),
        rows,
        k,
        weight.data_ptr(),
        n,
        out.data_ptr(),
        out.stride(0),
        epilogue,
        None,
        0,
        status_word(x.device).data_ptr(),
        _stream(x.device),
    )
    return out


class RowStats:
    """RMSNorm statistics of a residual stream handed from one GEMM to the next:
    ``x`` [T, D] fp32 (the un-rounded residual sum) and ``ss`` [parts, T] fp32
    (sums of squares over each 128-column tile, or over the whole row)."""

    __slots__ = ("x", "ss")

    def __init__(self, x: torch.Tensor, ss: torch.Tensor):
        self.x, self.ss = x, ss

    @classmethod
    def empty(cls, rows: int, hidden: int, parts: int, device: torch.device) -> "RowStats":
        return cls(torch.empty((rows, hidden), dtype=torch.float32, device=device),
                   torch.empty((parts, rows), dtype=torch.float32, device=device))

    @property
    def parts(self) -> int:
        return self.ss.shape[0]

    def rows(self, start: int, stop: int) -> "RowStats":
        return RowStats(self.x[start:stop], self.ss[:, start:stop])

    def select(self, idx: torch.Tensor) -> "RowStats":
        return RowStats(self.x.index_select(0, idx).contiguous(), self.ss.index_select(1, idx).contiguous())


def embedding_stat(ids: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, RowStats]:
    """Embedding rows plus their RMSNorm statistics (one part per row)."""
    _require_cuda(ids, weight, what="embedding_stat")
    ids = ids.contiguous()
    if ids.dtype not in (torch.int64, torch.int32):
        raise ValueError("embedding ids must be int32 or int64")
    t, d = ids.numel(), weight.shape[1]
    out = torch.empty((t, d), dtype=weight.dtype, device=weight.device)
    st = RowStats.empty(t, d, 1, weight.device)
    _lib.call("aiosb_embedding_stat", ids.data_ptr(), int(ids.dtype == torch.int64), t, weight.data_ptr(),
              weight.shape[0], d, out.data_ptr(), st.x.data_ptr(), st.ss.data_ptr(),
              status_word(ids.device).data_ptr(), _stream(ids.device))
    return out, st


def linear_add_stat(x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor) -> RowStats:
    """residual <- bf16(residual + bf16(x @ weight.T)) in place, returning the
    RMSNorm statistics of the new residual stream."""
    _require_cuda(x, weight, residual, what="linear_add_stat")
    if x.ndim != 2 or weight.ndim != 2 or x.shape[1] != weight.shape[1] or not x.is_contiguous():
        raise ValueError("linear_add_stat expects contiguous x [T, K] and weight [N, K]")
    rows, n = x.shape[0], weight.shape[0]
    if residual.shape != (rows, n) or residual.stride(1) != 1:
        raise ValueError("linear_add_stat needs a residual [rows, n] with contiguous rows")
    st = RowStats.empty(rows, n, n // 8, x.device)
    parts = ctypes.c_int64(0)
    _lib.call("aiosb_linear_add_stat", x.data_ptr(), rows, x.shape[1], weight.data_ptr(), n, residual.data_ptr(),
              residual.stride(0), residual.data_ptr(), residual.stride(0), st.x.data_ptr(), st.ss.data_ptr(),
              st.ss.stride(0), ctypes.byref(parts), status_word(x.device).data_ptr(), _stream(x.device))
    return RowStats(st.x, st.ss[: parts.value])


def linear_stat_norm(
    stats: RowStats,
    norm_weight: torch.Tensor,
    eps: float,
    weight: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    epilogue: int = _lib.EPI_STORE,
    tile_stats: torch.Tensor | None = None,
    early_dependents: bool = False,
) -> torch.Tensor:
    """``linear(rmsnorm(s) * norm_weight, weight)`` with s and its sums of squares
    from ``stats``; the normalised rows exist only inside the GEMM.
    ``early_dependents``: the next kernel may launch before this one's wait
    (``LINEAR_EARLY_DEPENDENTS``; the caller vouches for the successor). With
    ``tile_stats`` (fp32, [n / 16, rows, 4], see ``tile_stats_eligible``) the
    store epilogue also writes each 16-column tile's (max, sum of exp(v - max),
    min, NaN flag) of the stored values."""
    _require_cuda(stats.x, norm_weight, weight, what="linear_stat_norm")
    rows, k = stats.x.shape
    if weight.shape[1] != k or stats.x.stride(1) != 1 or stats.x.stride(0) != k or stats.ss.stride(1) != 1:
        raise ValueError("linear_stat_norm expects contiguous statistics [rows, k] matching the weight")
    n = weight.shape[0]
    cols = n // 2 if epilogue == _lib.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((rows, cols), dtype=weight.dtype, device=weight.device)
    if tile_stats is not None:
        _check_tile_stats(tile_stats, epilogue, rows, k, n)
        _lib.call("aiosb_linear_stat_norm_tiles", stats.x.data_ptr(), stats.ss.data_ptr(), stats.ss.stride(0),
                  stats.parts, norm_weight.data_ptr(), float(eps), rows, k, weight.data_ptr(), n, out.data_ptr(),
                  out.stride(0), tile_stats.data_ptr(), status_word(weight.device).data_ptr(),
                  _stream(weight.device))
        return out
    flags = _lib.LINEAR_EARLY_DEPENDENTS if early_dependents else 0
    _lib.call("aiosb_linear_stat_norm", stats.x.data_ptr(), stats.ss.data_ptr(), stats.ss.stride(0), stats.parts,
              norm_weight.data_ptr(), float(eps), rows, k, weight.data_ptr(), n, out.data_ptr(), out.stride(0),
              epilogue | flags, None, 0, status_word(weight.device).data_ptr(), _stream(weight.device))
    return out


def _check_tile_stats(tile_stats: torch.Tensor, epilogue: int, rows: int, k: int, n: int) -> None:
    if epilogue != _lib.EPI_STORE or not tile_stats_eligible(rows, k, n):
        raise ValueError("tile statistics need the store epilogue, rows <= 16, k <= 768, n % 16 == 0")
    if tile_stats.dtype != torch.float32 or not tile_stats.is_contiguous() or tile_stats.numel() < n // 16 * rows * 4:
        raise ValueError("tile_stats must be contiguous fp32 with n / 16 * rows * 4 elements")


def tile_stats_eligible(rows: int, k: int, n: int) -> bool:
    """Whether ``linear_stat_norm`` can write tile statistics for this shape (the
    library's answer: the register-operand path with rows <= 16, k a multiple of
    256 up to 768, n % 16 == 0)."""
    return bool(_lib.load().aiosb_linear_tile_stats_eligible(rows, k, n))


def pack_gate_up(weight: torch.Tensor) -> torch.Tensor:
    """[gate | up] rows ([2F, K]) -> 64-row interleaved blocks for EPI_SILU_MUL."""
    two_f, k = weight.shape
    f = two_f // 2
    if f % 64:
        raise ValueError("gate/up width must be a multiple of 64")
    gate = weight[:f].reshape(f // 64, 64, k)
    up = weight[f:].reshape(f // 64, 64, k)
    return torch.stack((gate, up), dim=1).reshape(two_f, k).contiguous()


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def attention_decode(
    *,
    out: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    page_table: torch.Tensor,
    row_table: torch.Tensor,
    seq_lens: torch.Tensor,
    positions: torch.Tensor,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    scale: float,
    qkv: torch.Tensor | None = None,
    q: torch.Tensor | None = None,
    q_norm_w: torch.Tensor | None = None,
    k_norm_w: torch.Tensor | None = None,
    eps: float = 1e-6,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    out_loc: torch.Tensor | None = None,
    prefix_len: torch.Tensor | None = None,
    active: torch.Tensor | None = None,
    stable_history: bool | int = False,
    staged_prefix: int = 0,
) -> torch.Tensor:
    """Decode attention. ``stable_history`` (fused ``qkv`` mode): the row table,
    prefix length, page-table entries before each row's current position and their
    K/V were written before the previous kernel on the stream began, so the kernel
    may stage them before waiting on that kernel. ``True`` / ``HISTORY_STAGED``:
    each row reads its keys itself; ``HISTORY_PREFIX_ONCE``: the rows of a KV head
    read the shared prefix once between them (a cluster of up to 8 rows).
    ``staged_prefix``: a bound on the prefix length (0: 128); the kernel stages that
    many prefix keys before its wait and sizes its shared memory by it."""
    rows = out.shape[0]
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    src = qkv if qkv is not None else q
    _lib.call(
        "aiosb_attention_decode",
        _ptr(qkv),
        qkv.stride(0) if qkv is not None else 0,
        _ptr(q),
        q.stride(0) if q is not None else 0,
        _ptr(q_norm_w),
        _ptr(k_norm_w),
        float(eps),
        _ptr(cos),
        _ptr(sin),
        cos.shape[0] if cos is not None else 0,
        positions.data_ptr(),
        _ptr(out_loc),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        num_slots,
        page_table.data_ptr(),
        page_table.stride(0),
        row_table.data_ptr(),
        seq_lens.data_ptr(),
        _ptr(prefix_len),
        _ptr(active),
        int(stable_history),
        int(staged_prefix),
        rows,
        num_qo_heads,
        num_kv_heads,
        head_dim,
        float(scale),
        out.data_ptr(),
        out.stride(0),
        status_word(src.device).data_ptr(),
        _stream(src.device),
    )
    return out


def qk_norm_rope_store(
    *,
    qkv: torch.Tensor,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    q_norm_w: torch.Tensor,
    k_norm_w: torch.Tensor,
    eps: float,
    cos: torch.Tensor,
    sin: torch.Tensor,
    positions: torch.Tensor,
    out_loc: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    q_out: torch.Tensor,
) -> torch.Tensor:
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    _lib.call(
        "aiosb_qk_norm_rope_store",
        qkv.data_ptr(),
        qkv.stride(0),
        qkv.shape[0],
        num_qo_heads,
        num_kv_heads,
        head_dim,
        q_norm_w.data_ptr(),
        k_norm_w.data_ptr(),
        float(eps),
        cos.data_ptr(),
        sin.data_ptr(),
        cos.shape[0],
        positions.data_ptr(),
        out_loc.data_ptr(),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        num_slots,
        q_out.data_ptr(),
        q_out.stride(0),
        status_word(qkv.device).data_ptr(),
        _stream(qkv.device),
    )
    return q_out


FUSED_PREFILL_MAX_TOKENS = 64  # new tokens per request on the fused prefill


def attention_prefill_fused(
    *,
    qkv: torch.Tensor,
    out: torch.Tensor,
    q_norm_w: torch.Tensor,
    k_norm_w: torch.Tensor,
    eps: float,
    cos: torch.Tensor,
    sin: torch.Tensor,
    positions: torch.Tensor,
    out_loc: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    page_table: torch.Tensor,
    meta: torch.Tensor,
    num_requests: int,
    num_tiles: int,
    tile_tokens: int,
    max_q_len: int,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    scale: float,
) -> torch.Tensor:
    """``qk_norm_rope_store`` and ``attention_prefill`` in one launch, for
    requests of at most FUSED_PREFILL_MAX_TOKENS new tokens whose cached keys were
    written by earlier launches; ``meta`` as for ``attention_prefill``. The output
    and the stored K/V equal the two-call path bit for bit."""
    _require_cuda(qkv, out, k_cache, v_cache, page_table, meta, what="attention_prefill_fused")
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    base = meta.data_ptr()
    r = num_requests * 4
    _lib.call(
        "aiosb_attention_prefill_fused",
        qkv.data_ptr(), qkv.stride(0), q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps),
        cos.data_ptr(), sin.data_ptr(), cos.shape[0], positions.data_ptr(), out_loc.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), num_slots, page_table.data_ptr(), page_table.stride(0),
        base, base + r, base + 2 * r, base + 3 * r, base + 4 * r, base + 4 * r + num_tiles * 4,
        num_tiles, tile_tokens, max_q_len, num_qo_heads, num_kv_heads, head_dim, float(scale),
        out.data_ptr(), out.stride(0), status_word(qkv.device).data_ptr(), _stream(qkv.device),
    )
    return out


def prefill_tile_tokens(num_qo_heads: int, num_kv_heads: int) -> int:
    n = _lib.load().aiosb_prefill_tile_tokens(num_qo_heads, num_kv_heads)
    if n <= 0:
        raise ValueError("unsupported head grouping for prefill attention")
    return n


def attention_prefill(
    *,
    q: torch.Tensor,
    out: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    page_table: torch.Tensor,
    meta: torch.Tensor,
    num_requests: int,
    num_tiles: int,
    tile_tokens: int,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    scale: float,
) -> torch.Tensor:
    """``meta`` is one int32 device tensor holding, back to back, the request
    arrays q_start, q_len, cached_len, table_row ([num_requests] each) and the
    tile arrays tile_req, tile_q0 ([num_tiles] each)."""
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    base = meta.data_ptr()
    r = num_requests * 4
    _lib.call(
        "aiosb_attention_prefill",
        q.data_ptr(),
        q.stride(0),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        num_slots,
        page_table.data_ptr(),
        page_table.stride(0),
        base,
        base + r,
        base + 2 * r,
        base + 3 * r,
        base + 4 * r,
        base + 4 * r + num_tiles * 4,
        num_tiles,
        tile_tokens,
        num_qo_heads,
        num_kv_heads,
        head_dim,
        float(scale),
        out.data_ptr(),
        out.stride(0),
        status_word(q.device).data_ptr(),
        _stream(q.device),
    )
    return out


def prefill_meta(
    q_lens: list[int], cached_lens: list[int], table_rows: list[int], tile_tokens: int
) -> tuple[list[int], int]:
    """Host-side request/tile arrays for :func:`attention_prefill`."""
    q_start, acc = [], 0
    tile_req, tile_q0 = [], []
    for i, n in enumerate(q_lens):
        q_start.append(acc)
        acc += n
        for q0 in range(0, n, tile_tokens):
            tile_req.append(i)
            tile_q0.append(q0)
    return [*q_start, *q_lens, *cached_lens, *table_rows, *tile_req, *tile_q0], len(tile_req)


# ---------------------------------------------------------------------------
# Sampler / uniforms / slot FIFO
# ---------------------------------------------------------------------------
def sample(
    logits: torch.Tensor,
    *,
    temperature: float,
    top_k: int,
    top_p: float,
    greedy: bool,
    uniforms: torch.Tensor | None,
    forbidden: torch.Tensor | None = None,
    forbidden_rows: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    rows, vocab = logits.shape
    dev = logits.device
    tok = torch.empty((rows, 1), dtype=torch.int64, device=dev)
    lp = torch.empty((rows, 1), dtype=torch.float32, device=dev)
    _lib.call(
        "aiosb_sample",
        logits.data_ptr(),
        rows,
        vocab,
        logits.stride(0),
        float(temperature),
        int(top_k),
        float(top_p),
        int(bool(greedy)),
        _ptr(uniforms),
        _ptr(forbidden),
        0 if forbidden is None else forbidden.numel(),
        _ptr(forbidden_rows),
        0 if forbidden_rows is None else forbidden_rows.shape[1],
        tok.data_ptr(),
        lp.data_ptr(),
        status_word(dev).data_ptr(),
        _stream(dev),
    )
    return tok, lp


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """log_softmax(logits.float())[r, targets[r]] per row, fp32."""
    rows, vocab = logits.shape
    t = targets.to(device=logits.device, dtype=torch.int64).contiguous()
    out = torch.empty(rows, dtype=torch.float32, device=logits.device)
    _lib.call("aiosb_token_logprobs", logits.data_ptr(), rows, vocab, logits.stride(0), t.data_ptr(),
              out.data_ptr(), status_word(logits.device).data_ptr(), _stream(logits.device))
    return out


def stateless_uniforms_device(seeds: torch.Tensor, steps: int) -> torch.Tensor:
    out = torch.empty((seeds.numel(), steps), dtype=torch.float32, device=seeds.device)
    _lib.call("aiosb_stateless_uniforms", seeds.data_ptr(), seeds.numel(), steps, out.data_ptr(), _stream(seeds.device))
    return out


def slot_alloc(ring: torch.Tensor, head: int, n: int) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.int32, device=ring.device)
    _lib.call("aiosb_slot_alloc", ring.data_ptr(), ring.numel(), head, n, out.data_ptr(), _stream(ring.device))
    return out


def slot_free(ring: torch.Tensor, tail: int, slots: torch.Tensor) -> None:
    slots = slots.to(torch.int32).contiguous()
    _lib.call("aiosb_slot_free", ring.data_ptr(), ring.numel(), tail, slots.data_ptr(), slots.numel(), _stream(ring.device))


def slot_free_range(ring: torch.Tensor, begin: int, n: int, tail: int) -> None:
    _lib.call("aiosb_slot_free_range", ring.data_ptr(), ring.numel(), begin, n, tail, _stream(ring.device))
