"""aiosb_group_step_static, the CandidateGroup step for callers that cannot
allocate device memory, against aiosb_group_step.

Some hosts of this library cannot call cudaMalloc: a plugin whose host process
owns all device memory through its own allocator and hands the plugin only the
buffers it needs, or a per-keystroke path that cannot afford the device
synchronisation of a cudaMalloc / cudaFree pair. For them the step keeps its
per-row finish flags in a fixed 32-entry array inside the library instead of the
caller's `finished` buffer. This test drives two identical groups through the
C ABI, one with each entry point, and checks that two steps in a row leave
identical results: sampled ids, log-probabilities, stop codes, the compaction of
finished rows, the FIFO slots and page-table entries, and the group state.

The file is named to be collected last, so a run that stops at its first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from aios_b200 import _lib

pytestmark = pytest.mark.gpu

ROWS = 8
VOCAB = 16384
STEPS = 4
TABLE_WIDTH = 64
CAPACITY = 256
PREFIX_LEN = 5
EOS, PAD, TERMINAL = 2, 0, 7


def _make_group(dev: torch.device) -> dict:
    i32 = dict(dtype=torch.int32, device=dev)
    b = dict(
        state=torch.zeros(ctypes.sizeof(_lib.GroupState), dtype=torch.uint8, device=dev),
        logits=torch.zeros((ROWS, VOCAB), dtype=torch.bfloat16, device=dev),
        uniforms=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        output_ids=torch.zeros((ROWS, STEPS), **i32),
        token_logprobs=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        logprob_sums=torch.zeros(ROWS, dtype=torch.float32, device=dev),
        terminal_ids=torch.tensor([TERMINAL], **i32),
        page_table=torch.zeros((ROWS, TABLE_WIDTH), **i32),
        ring=torch.arange(CAPACITY, **i32),
        status=torch.zeros(1, **i32),
    )
    for name in ("counts", "stop_codes", "active", "finished", "tokens", "positions", "seq_lens", "out_loc",
                 "row_page", "row_table"):
        b[name] = torch.zeros(ROWS, **i32)
    st = _lib.GroupState(
        step=0, max_steps=STEPS, min_new_tokens=0, prefix_len=PREFIX_LEN, row_offset=0, rows=ROWS, vocab=VOCAB,
        eos_id=EOS, pad_id=PAD, greedy=0, top_k=50, temperature=0.8, top_p=0.9, page_size=1, n_terminal=1,
        head=0, tail=CAPACITY, capacity=CAPACITY, table_stride=TABLE_WIDTH,
    )
    b["state"].copy_(torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8))
    fields = {name for name, _ in _lib.GroupPtrs._fields_}
    b["ptrs"] = _lib.GroupPtrs(**{k: v.data_ptr() for k, v in b.items() if k in fields})
    return b


def _results(b: dict) -> dict:
    names = ("output_ids", "token_logprobs", "counts", "logprob_sums", "stop_codes", "active", "tokens",
             "positions", "seq_lens", "out_loc", "page_table", "state", "status")
    return {k: b[k].cpu().clone() for k in names}


def _logits(gen: torch.Generator, dev: torch.device, eos_rows: list[int], terminal_rows: list[int]) -> torch.Tensor:
    x = torch.randn((ROWS, VOCAB), generator=gen)
    x[:, [EOS, TERMINAL]] = -20.0  # never sampled, except where raised below
    x[eos_rows, EOS] = 20.0  # sampled with probability ~1 at temperature 0.8
    x[terminal_rows, TERMINAL] = 20.0
    return x.to(dev, torch.bfloat16)


def test_group_step_static_matches_group_step(cuda_device) -> None:
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    gen = torch.Generator().manual_seed(0)
    prefix_logits = torch.randn(VOCAB, generator=gen).to(dev, torch.bfloat16)
    ref, nal = _make_group(dev), _make_group(dev)
    for g in (ref, nal):
        _lib.call("aiosb_group_begin", ctypes.byref(g["ptrs"]), prefix_logits.data_ptr(), 1234, ROWS, ROWS, stream)
    # the allocation-free caller has no `finished` array: the entry point must not touch it
    nal_ptrs = _lib.GroupPtrs.from_buffer_copy(nal["ptrs"])
    nal_ptrs.finished = None
    # step 0: rows 1 and 5 end on EOS, row 3 on a terminal id; step 1: row 6 ends on EOS
    for step, (eos_rows, term_rows) in enumerate([([1, 5], [3]), ([6], [])]):
        logits = _logits(gen, dev, eos_rows, term_rows)
        ref["logits"].copy_(logits)
        nal["logits"].copy_(logits)
        _lib.call("aiosb_group_step", ctypes.byref(ref["ptrs"]), ROWS, VOCAB, 50, stream)
        _lib.call("aiosb_group_step_static", ctypes.byref(nal_ptrs), ROWS, VOCAB, 50, stream)
        torch.cuda.synchronize(dev)
        want, got = _results(ref), _results(nal)
        # the same kernel on the same inputs: every output is bit-identical
        for name in want:
            torch.testing.assert_close(got[name], want[name], rtol=0, atol=0, msg=f"step {step}: {name}")
        assert int(want["status"][0]) == 0
        state = _lib.GroupState.from_buffer_copy(bytes(want["state"].numpy()))
        assert state.step == step + 1 and state.done == 0 and state.arrive == 0
    # the finished rows were compacted out, the others got consecutive FIFO slots
    assert want["stop_codes"].tolist() == [0, 1, 0, 2, 0, 1, 1, 0]
    assert want["active"].tolist() == [1, 0, 1, 0, 1, 0, 0, 1]
    assert want["out_loc"][[0, 2, 4, 7]].tolist() == [5, 6, 7, 8]
    assert nal["finished"].abs().sum().item() == 0


def test_group_step_static_rejects_rows_beyond_its_array(cuda_device) -> None:
    g = _make_group(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    with pytest.raises(ValueError, match="33 rows exceed the 32-row static scratch"):
        _lib.call("aiosb_group_step_static", ctypes.byref(g["ptrs"]), 33, VOCAB, 50, stream)
