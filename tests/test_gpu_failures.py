"""Failures made on the host, seen through the status word, with the GPU context
still usable afterwards (no fault, trap or hang is caused on the device).

* Pool exhaustion: a group step whose free-slot FIFO holds fewer entries than
  the rows that survive the step reports AIOSB_DEV_POOL_EMPTY, ends the group
  (done) instead of handing out slots it does not have, and the next group on a
  sufficient pool steps normally. The reference raises NotImplementedError in
  the same situation on the host (aios/scheduler/cache.py:46-51); the device
  step cannot raise, so it stops the group and reports.
* A bounded mbarrier wait that runs out: the mixer's stream kernel with a
  test hook that announces one tile without copying it (nothing is in flight,
  so nothing can fault) and a 2 ms wait bound reports AIOSB_DEV_WAIT_TIMEOUT,
  writes NaN into the rows it could not mix, and the next launch without the
  hook is exact again.
* The decode-step bounded flag wait is covered by tests/test_gpu_decode_step.py.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from aios_b200 import _lib

pytestmark = pytest.mark.gpu

ROWS, VOCAB, STEPS, WIDTH = 8, 16384, 4, 64


def _group(dev: torch.device, free: int) -> dict:
    i32 = dict(dtype=torch.int32, device=dev)
    b = dict(
        state=torch.zeros(ctypes.sizeof(_lib.GroupState), dtype=torch.uint8, device=dev),
        logits=torch.randn((ROWS, VOCAB), generator=torch.Generator().manual_seed(1)).to(dev, torch.bfloat16),
        uniforms=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        output_ids=torch.zeros((ROWS, STEPS), **i32),
        token_logprobs=torch.zeros((ROWS, STEPS), dtype=torch.float32, device=dev),
        logprob_sums=torch.zeros(ROWS, dtype=torch.float32, device=dev),
        terminal_ids=torch.tensor([7], **i32),
        page_table=torch.zeros((ROWS, WIDTH), **i32),
        ring=torch.arange(64, **i32),
        status=torch.zeros(1, **i32),
    )
    b["logits"][:, [2, 7]] = -20.0  # no row stops on EOS or the terminal id: all 8 need a slot
    for name in ("counts", "stop_codes", "active", "finished", "tokens", "positions", "seq_lens", "out_loc",
                 "row_page", "row_table"):
        b[name] = torch.zeros(ROWS, **i32)
    st = _lib.GroupState(step=0, max_steps=STEPS, prefix_len=5, rows=ROWS, vocab=VOCAB, eos_id=2, pad_id=0,
                         top_k=50, temperature=0.8, top_p=0.9, page_size=1, n_terminal=1, head=0, tail=free,
                         capacity=64, table_stride=WIDTH)
    b["state"].copy_(torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8))
    fields = {name for name, _ in _lib.GroupPtrs._fields_}
    b["ptrs"] = _lib.GroupPtrs(**{k: v.data_ptr() for k, v in b.items() if k in fields})
    return b


def _step(dev: torch.device, g: dict) -> _lib.GroupState:
    stream = torch.cuda.current_stream(dev).cuda_stream
    prefix = g["logits"][0].clone()
    _lib.call("aiosb_group_begin", ctypes.byref(g["ptrs"]), prefix.data_ptr(), 99, ROWS, ROWS, stream)
    _lib.call("aiosb_group_step", ctypes.byref(g["ptrs"]), ROWS, VOCAB, 50, stream)
    torch.cuda.synchronize(dev)
    return _lib.GroupState.from_buffer_copy(bytes(g["state"].cpu().numpy()))


def test_exhausted_free_list_reports_pool_empty_and_ends_the_group(cuda_device) -> None:
    short = _group(cuda_device, free=3)  # 8 rows survive the first step, 3 slots are free
    st = _step(cuda_device, short)
    assert int(short["status"][0]) == _lib.DEV_POOL_EMPTY
    assert st.done == 1 and st.head == 0  # nothing was handed out
    assert int(short["out_loc"].max()) < 0 or bool((short["out_loc"] == -1).all())
    # the context still works: the same step on a pool that suffices
    ok = _group(cuda_device, free=64)
    st = _step(cuda_device, ok)
    assert int(ok["status"][0]) == 0
    assert st.done == 0 and st.head == ROWS  # one slot per row, in FIFO order
    assert ok["out_loc"].tolist() == list(range(ROWS))


def test_mixer_stream_wait_that_runs_out_reports_and_recovers(cuda_device) -> None:
    from aios_b200.kernel import ops

    g = torch.Generator(device=cuda_device).manual_seed(5)
    tokens = 4096  # the stream kernel (from 2048 tokens)
    bank = torch.randn(4, tokens, 768, generator=g, device=cuda_device).to(torch.bfloat16)
    part = torch.randn(tokens, 768, generator=g, device=cuda_device).to(torch.bfloat16)
    wq = torch.randn(768, generator=g, device=cuda_device) * 0.02
    good = ops.b200_attnres_mix(bank, part, wq, 1e-6)
    torch.cuda.synchronize(cuda_device)
    ops.check_status(cuda_device)
    _lib.call("aiosb_test_attnres_stream_stall", 0, 2_000_000)
    try:
        bad = ops.b200_attnres_mix(bank, part, wq, 1e-6)
        torch.cuda.synchronize(cuda_device)
    finally:
        _lib.call("aiosb_test_attnres_stream_stall", -1, 0)
    with pytest.raises(RuntimeError, match="wait"):
        ops.check_status(cuda_device)
    assert bool(torch.isnan(bad[:4].float()).all())  # CTA 0's first tile was never mixed
    again = ops.b200_attnres_mix(bank, part, wq, 1e-6)
    torch.cuda.synchronize(cuda_device)
    ops.check_status(cuda_device)
    assert torch.equal(again, good)
