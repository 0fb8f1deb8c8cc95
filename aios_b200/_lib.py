"""ctypes binding of the C ABI in ``include/aios_b200.h`` (``libaios_b200.so``).

This module is the only place that touches raw addresses: every wrapper in
``aios_b200.kernel.ops`` passes ``tensor.data_ptr()`` values, sizes and the current
CUDA stream through the functions declared here. A missing library is an error;
there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libaios_b200.so"

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_MISALIGNED = -3
ERR_LAUNCH = -4

DEV_WAIT_TIMEOUT = 1
DEV_SLOT_RANGE = 2
DEV_TOKEN_RANGE = 3
DEV_POOL_EMPTY = 4
DEV_POSITION_RANGE = 5

DEVICE_STATUS_NAMES = {
    DEV_WAIT_TIMEOUT: "a bounded device wait ran out",
    DEV_SLOT_RANGE: "KV slot index outside the pool",
    DEV_TOKEN_RANGE: "token id outside the vocabulary",
    DEV_POOL_EMPTY: "free-slot FIFO exhausted",
    DEV_POSITION_RANGE: "position outside the RoPE table",
}

EPI_STORE = 0
EPI_SILU_MUL = 1
EPI_ADD = 2
LINEAR_EARLY_DEPENDENTS = 0x100  # OR-ed into a linear's epilogue (aios_b200.h)
GROUP_AFTER_FORWARD = 1  # aiosb_group_ptrs.flags
HISTORY_STAGED = 1  # aiosb_attention_decode stable_history modes
HISTORY_PREFIX_ONCE = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64


class GroupState(ctypes.Structure):
    """Mirror of ``aiosb_group_state``."""

    _fields_ = [
        ("step", _i32),
        ("max_steps", _i32),
        ("min_new_tokens", _i32),
        ("prefix_len", _i32),
        ("row_offset", _i32),
        ("rows", _i32),
        ("vocab", _i32),
        ("eos_id", _i32),
        ("pad_id", _i32),
        ("greedy", _i32),
        ("top_k", _i32),
        ("temperature", _f32),
        ("top_p", _f32),
        ("page_size", _i32),
        ("n_terminal", _i32),
        ("n_minlen", _i32),
        ("n_banned", _i32),
        ("banned_width", _i32),
        ("ban_min_prefix", _i32),
        ("done", _i32),
        ("cancelled", _i32),
        ("n_active", _i32),
        ("active_model_tokens", _i32),
        ("arrive", _i32),
        ("head", _i64),
        ("tail", _i64),
        ("capacity", _i64),
        ("table_stride", _i64),
    ]


class GroupPtrs(ctypes.Structure):
    """Mirror of ``aiosb_group_ptrs`` (device addresses)."""

    _fields_ = [
        ("state", _p),
        ("cancel_flag", _p),
        ("host_mirror", _p),
        ("logits", _p),
        ("uniforms", _p),
        ("output_ids", _p),
        ("token_logprobs", _p),
        ("counts", _p),
        ("logprob_sums", _p),
        ("stop_codes", _p),
        ("active", _p),
        ("finished", _p),
        ("tokens", _p),
        ("positions", _p),
        ("seq_lens", _p),
        ("out_loc", _p),
        ("row_page", _p),
        ("row_table", _p),
        ("terminal_ids", _p),
        ("minlen_ids", _p),
        ("banned", _p),
        ("banned_len", _p),
        ("page_table", _p),
        ("ring", _p),
        ("status", _p),
        ("tile_stats", _p),
        ("flags", _i64),
        ("embed_w", _p),
        ("embed_out", _p),
        ("embed_stat_x", _p),
        ("embed_stat_ss", _p),
        ("hidden", _i64),
    ]


class DecodeLayer(ctypes.Structure):
    """Mirror of ``aiosb_decode_layer`` (device addresses)."""

    _fields_ = [(name, _p) for name in ("w_qkv", "w_o", "w_gate_up", "w_down", "in_norm", "post_norm", "q_norm",
                                        "k_norm", "k_cache", "v_cache")]


class DecodeStepArgs(ctypes.Structure):
    """Mirror of ``aiosb_decode_step_args``."""

    _fields_ = [
        ("layers", _p),
        ("num_layers", _i32), ("rows", _i32), ("hidden", _i32), ("intermediate", _i32), ("num_qo_heads", _i32),
        ("num_kv_heads", _i32), ("head_dim", _i32), ("vocab", _i32),
        ("eps", _f32), ("scale", _f32),
        ("embed", _p), ("final_norm", _p), ("lm_head", _p),
        ("tokens", _p), ("positions", _p), ("out_loc", _p), ("row_table", _p), ("seq_lens", _p),
        ("prefix_len", _p), ("active", _p), ("page_table", _p),
        ("table_stride", _i64), ("num_slots", _i64),
        ("cos_tab", _p), ("sin_tab", _p), ("max_pos", _i32),
        ("work", _p), ("logits", _p), ("logits_stride", _i64),
        ("sync", _p), ("status", _p), ("wait_limit_ns", _u64), ("test_flag_skew", ctypes.c_uint32),
        ("grid_ctas", _i32),
    ]


_SIGNATURES = {
    "aiosb_version": ([], _i32),
    "aiosb_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _i32),
    "aiosb_host_device_pointer": ([_p, ctypes.POINTER(_p)], _i32),
    "aiosb_kv_store": ([_p, _p, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _p, _p], _i32),
    "aiosb_attnres_mix": ([_p, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _p], _i32),
    "aiosb_attnres_mix_rmsnorm": ([_p, _i64, _i64, _i64, _p, _p, _f32, _p, _f32, _i64, _p, _p], _i32),
    "aiosb_test_attnres_stream_stall": ([_i64, ctypes.c_uint64], _i32),
    "aiosb_linear_tile_stats_eligible": ([_i64, _i64, _i64], _i32),
    "aiosb_linear_tiles": ([_p, _i64, _i64, _p, _i64, _p, _i64, _p, _p, _p], _i32),
    "aiosb_linear_stat_norm_tiles": (
        [_p, _p, _i64, _i64, _p, _f32, _i64, _i64, _p, _i64, _p, _i64, _p, _p, _p], _i32
    ),
    "aiosb_linear_attnres_rmsnorm": (
        [_p, _i64, _i64, _i64, _p, _p, _f32, _p, _f32, _p, _i64, _i64, _p, _i64, _i32, _p, _p], _i32
    ),
    "aiosb_rmsnorm": ([_p, _i64, _i64, _i64, _i64, _p, _f32, _p, _i64, _p], _i32),
    "aiosb_add_rmsnorm": ([_p, _p, _i64, _i64, _p, _f32, _p], _i32),
    "aiosb_silu_mul": ([_p, _i64, _i64, _p, _p], _i32),
    "aiosb_embedding": ([_p, _i32, _i64, _p, _i64, _i64, _p, _p, _p], _i32),
    "aiosb_embedding_stat": ([_p, _i32, _i64, _p, _i64, _i64, _p, _p, _p, _p, _p], _i32),
    "aiosb_linear": ([_p, _i64, _i64, _p, _i64, _p, _i64, _i32, _p, _i64, _p, _p], _i32),
    "aiosb_linear_rmsnorm": (
        [_p, _p, _p, _p, _f32, _i64, _i64, _p, _i64, _p, _i64, _i32, _p, _i64, _p, _p], _i32
    ),
    "aiosb_linear_add_stat": ([_p, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _p, _p, _p], _i32),
    "aiosb_linear_stat_norm": (
        [_p, _p, _i64, _i64, _p, _f32, _i64, _i64, _p, _i64, _p, _i64, _i32, _p, _i64, _p, _p], _i32
    ),
    "aiosb_attention_decode": (
        [_p, _i64, _p, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p, _p, _p, _i32,
         _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _p, _p],
        _i32,
    ),
    "aiosb_qk_norm_rope_store": (
        [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p],
        _i32,
    ),
    "aiosb_prefill_tile_tokens": ([_i64, _i64], _i32),
    "aiosb_attention_prefill": (
        [_p, _i64, _p, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64,
         _p, _p],
        _i32,
    ),
    "aiosb_attention_prefill_fused": (
        [_p, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64,
         _i64, _i64, _i64, _i64, _f32, _p, _i64, _p, _p],
        _i32,
    ),
    "aiosb_sample": (
        [_p, _i64, _i64, _i64, _f32, _i64, _f32, _i32, _p, _p, _i64, _p, _i64, _p, _p, _p, _p],
        _i32,
    ),
    "aiosb_stateless_uniforms": ([_p, _i64, _i64, _p, _p], _i32),
    "aiosb_page_table_fill": ([_p, _i64, _i64, _i64, _p, _i64, _p], _i32),
    "aiosb_token_logprobs": ([_p, _i64, _i64, _i64, _p, _p, _p, _p], _i32),
    "aiosb_slot_alloc": ([_p, _i64, _i64, _i64, _p, _p], _i32),
    "aiosb_slot_free": ([_p, _i64, _i64, _p, _i64, _p], _i32),
    "aiosb_slot_free_range": ([_p, _i64, _i64, _i64, _i64, _p], _i32),
    "aiosb_group_begin": ([ctypes.POINTER(GroupPtrs), _p, _u64, _i64, _i64, _p], _i32),
    "aiosb_group_step": ([ctypes.POINTER(GroupPtrs), _i64, _i64, _i64, _p], _i32),
    "aiosb_group_step_static": ([ctypes.POINTER(GroupPtrs), _i64, _i64, _i64, _p], _i32),
    "aiosb_decode_step_sync_words": ([], _i64),
    "aiosb_decode_step_work_bytes": ([_i64, _i64, _i64], _i64),
    "aiosb_decode_step": ([ctypes.POINTER(DecodeStepArgs), _p], _i32),
}

EXPORTED = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once and attaches the C signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("AIOS_B200_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"aios_b200 native library not found at {path}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` or `python -m aios_b200.build`"
            )
        lib = ctypes.CDLL(str(path))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().aiosb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Maps a C-ABI return code to the exception the reference raises."""
    if rc == OK:
        return
    msg = last_error()
    if rc in (ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_MISALIGNED):
        raise ValueError(msg or f"{what}: invalid argument ({rc})")
    raise RuntimeError(msg or f"{what}: launch failed ({rc})")


# Entry points that launch kernels; `launches` counts their successful calls
# (the bench reports it as the number of this library's kernel launches).
_NON_LAUNCHING = frozenset({"aiosb_version", "aiosb_last_error", "aiosb_host_device_pointer",
                            "aiosb_prefill_tile_tokens", "aiosb_decode_step_sync_words",
                            "aiosb_decode_step_work_bytes", "aiosb_linear_tile_stats_eligible"})
launches = 0


def call(name: str, *args) -> None:
    global launches
    check(getattr(load(), name)(*args), name)
    if name not in _NON_LAUNCHING:
        launches += 1


def count_launches(n: int = 1) -> None:
    global launches
    launches += n
