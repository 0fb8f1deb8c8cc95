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

ROWS = 8  # the bench's candidate group
MAX_ROWS = 32  # the static array's size: the largest group the entry point steps
VOCAB = 16384
STEPS = 4
TABLE_WIDTH = 64
CAPACITY = 256
PREFIX_LEN = 5
EOS, PAD, TERMINAL = 2, 0, 7


def _make_group(dev: torch.device, rows: int = ROWS) -> dict:
    i32 = dict(dtype=torch.int32, device=dev)
    b = dict(
        state=torch.zeros(ctypes.sizeof(_lib.GroupState), dtype=torch.uint8, device=dev),
        logits=torch.zeros((rows, VOCAB), dtype=torch.bfloat16, device=dev),
        uniforms=torch.zeros((rows, STEPS), dtype=torch.float32, device=dev),
        output_ids=torch.zeros((rows, STEPS), **i32),
        token_logprobs=torch.zeros((rows, STEPS), dtype=torch.float32, device=dev),
        logprob_sums=torch.zeros(rows, dtype=torch.float32, device=dev),
        terminal_ids=torch.tensor([TERMINAL], **i32),
        page_table=torch.zeros((rows, TABLE_WIDTH), **i32),
        ring=torch.arange(CAPACITY, **i32),
        status=torch.zeros(1, **i32),
    )
    for name in ("counts", "stop_codes", "active", "finished", "tokens", "positions", "seq_lens", "out_loc",
                 "row_page", "row_table"):
        b[name] = torch.zeros(rows, **i32)
    st = _lib.GroupState(
        step=0, max_steps=STEPS, min_new_tokens=0, prefix_len=PREFIX_LEN, row_offset=0, rows=rows, vocab=VOCAB,
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


def _logits(gen: torch.Generator, dev: torch.device, rows: int, eos_rows: list[int],
            terminal_rows: list[int]) -> torch.Tensor:
    x = torch.randn((rows, VOCAB), generator=gen)
    x[:, [EOS, TERMINAL]] = -20.0  # never sampled, except where raised below
    x[eos_rows, EOS] = 20.0  # sampled with probability ~1 at temperature 0.8
    x[terminal_rows, TERMINAL] = 20.0
    return x.to(dev, torch.bfloat16)


# (rows, [(eos rows, terminal rows) per step]): the bench's 8-row group and the
# 32-row maximum the static array holds
GROUPS = [
    (ROWS, [([1, 5], [3]), ([6], [])]),
    (MAX_ROWS, [([1, 5, 17, 30], [3, 31]), ([6, 20], [0])]),
]


@pytest.mark.parametrize("rows,endings", GROUPS, ids=[f"rows{g[0]}" for g in GROUPS])
def test_group_step_static_matches_group_step(cuda_device, rows, endings) -> None:
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    gen = torch.Generator().manual_seed(rows)
    prefix_logits = torch.randn(VOCAB, generator=gen).to(dev, torch.bfloat16)
    ref, nal = _make_group(dev, rows), _make_group(dev, rows)
    # the allocation-free caller has no `finished` array: neither the round start
    # nor the step may touch it
    nal_ptrs = _lib.GroupPtrs.from_buffer_copy(nal["ptrs"])
    nal_ptrs.finished = None
    nal["finished"].fill_(-7)  # would show any write through a stale pointer
    _lib.call("aiosb_group_begin", ctypes.byref(ref["ptrs"]), prefix_logits.data_ptr(), 1234, rows, rows, stream)
    _lib.call("aiosb_group_begin", ctypes.byref(nal_ptrs), prefix_logits.data_ptr(), 1234, rows, rows, stream)
    ended: dict[int, int] = {}
    for step, (eos_rows, term_rows) in enumerate(endings):
        logits = _logits(gen, dev, rows, eos_rows, term_rows)
        ref["logits"].copy_(logits)
        nal["logits"].copy_(logits)
        _lib.call("aiosb_group_step", ctypes.byref(ref["ptrs"]), rows, VOCAB, 50, stream)
        _lib.call("aiosb_group_step_static", ctypes.byref(nal_ptrs), rows, VOCAB, 50, stream)
        torch.cuda.synchronize(dev)
        want, got = _results(ref), _results(nal)
        # the same kernel on the same inputs: every output is bit-identical
        for name in want:
            torch.testing.assert_close(got[name], want[name], rtol=0, atol=0, msg=f"step {step}: {name}")
        assert int(want["status"][0]) == 0
        state = _lib.GroupState.from_buffer_copy(bytes(want["state"].numpy()))
        assert state.step == step + 1 and state.done == 0 and state.arrive == 0
        ended.update({r: 1 for r in eos_rows})
        ended.update({r: 2 for r in term_rows})
    # the finished rows were compacted out, the others got consecutive FIFO slots
    live = [r for r in range(rows) if r not in ended]
    assert want["stop_codes"].tolist() == [ended.get(r, 0) for r in range(rows)]
    assert want["active"].tolist() == [0 if r in ended else 1 for r in range(rows)]
    # step 0 took one slot per row that survived it (ring entries 0, 1, ...), so
    # the last step's slots continue from there
    first = rows - len(set(endings[0][0] + endings[0][1]))
    assert want["out_loc"][live].tolist() == list(range(first, first + len(live)))
    assert (nal["finished"] == -7).all(), "the NULL finished array was written"


def test_group_step_static_rejects_rows_beyond_its_array(cuda_device) -> None:
    g = _make_group(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    with pytest.raises(ValueError, match="33 rows exceed the 32-row static scratch"):
        _lib.call("aiosb_group_step_static", ctypes.byref(g["ptrs"]), 33, VOCAB, 50, stream)
