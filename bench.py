"""Benchmark of the B200 CandidateGroup keystroke (one JSON line on rank 0).

Workload (one "step" = one keystroke through the public API
``ImeCompletionEngine.complete``): the 0.1B-shaped MiniMind-IME model (S10: 14
layers, hidden 768, 12 q / 4 kv heads of 64, vocab 16384) with seeded random
weights, a fresh [BOS] + 12-token prefix per keystroke (ids uniform over the
CJK range, seeded), 8 candidates x 12 decode tokens at temperature 0.8,
top-k 50, top-p 0.9, one round (no refill), KV in 16-token pages of a 256-page
pool. Every keystroke prefills its prefix from scratch and streams the 201 MB of
weights once per decode step, so the working set exceeds the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

``--impl reference`` times the unmodified reference engine (installed under
baseline/_ref; fp32, all host cores, CPU shims for FlashInfer and the KV buffer)
on the same workload. With N > 1 (torchrun)
every GPU serves an independent keystroke stream (replicas; no data exchange);
the barrier and the max-over-ranks timing reduction run over gloo on host
values (no collective touches the GPUs), and each rank is pinned to its own
share of the host cores.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


def percentile(values, q):
    ordered = sorted(values)
    return ordered[max(0, min(len(ordered) - 1, math.ceil(q * len(ordered)) - 1))]


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, index: int, interval_ms: int = 50):
        self.index = index
        self.interval_ms = interval_ms
        self.samples: list[list[str]] = []
        self._proc = None
        self._mark = 0

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except OSError:
            self._proc = None
            return self
        # nvidia-smi's start-up (its NVML initialisation) stalls the GPU's work
        # for a while: the timed region starts only once it samples
        deadline = time.perf_counter() + 10.0
        while not self.samples and self._proc.poll() is None and time.perf_counter() < deadline:
            time.sleep(0.005)
        return self

    def mark(self) -> None:
        """Start of the timed region: the summary keeps the samples taken after it."""
        self._mark = len(self.samples)

    def _read(self):
        for line in self._proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self) -> dict:
        rows = [s for s in self.samples[self._mark:] if len(s) >= 8] or [s for s in self.samples if len(s) >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [v for v in (num(r[0]) for r in rows) if v is not None]
        reasons = set()
        for r in rows:
            for name, col in (("hw_slowdown", 4), ("hw_thermal_slowdown", 5), ("sw_thermal_slowdown", 6),
                              ("sw_power_cap", 7)):
                if r[col].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][1]),
                "reasons": sorted(reasons), "samples": len(rows)}


WORKLOAD = ("S10 keystroke: [BOS]+12 prefix, 8 candidates x 12 tokens, T=0.8 top-k 50 top-p 0.9, "
            "one round, 16-token pages x 256")


def bench_config(world: int) -> dict:
    """The `config` of both arms' lines (same workload, same keys)."""
    return {"workload": WORKLOAD, "model": "MiniMind-IME 0.1B shape (S10)", "prefix_tokens": 13,
            "candidates": 8, "max_new_tokens": 12, "page_size": 16, "num_pages": 256,
            "l2": "inputs larger than L2: every decode step streams the 201 MB of weights",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}


def keystroke_config():
    from aios_b200 import ImeGenerationConfig

    return ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                               max_new_tokens=12, temperature=0.8, top_k=50, top_p=0.9, seed=0)


def prefixes(tokenizer, vocab: int, count: int, seed: int, length: int = 12) -> list[str]:
    g = torch.Generator().manual_seed(seed)
    return [tokenizer.text_for(torch.randint(10, vocab, (length,), generator=g).tolist()) for _ in range(count)]


# ---------------------------------------------------------------------------
# Reference arm: the unmodified reference engine on the host cores
# ---------------------------------------------------------------------------
def run_reference(keystrokes: int, warmup: int, seed: int = 1234) -> dict:
    """Times the reference's own ``ImeCompletionEngine.complete`` (aios/ime.py:415-640,
    installed under baseline/_ref, fp32, all host threads) on the bench workload:
    the same seeded prefixes and the same weights rule as the GPU arm, one-token
    pages (the reference's only mode) over the same 4096 KV slots. The four CPU
    shims of oracle/reference_run.py stand in for FlashInfer and the CUDA-only KV
    buffer; this process imports nothing from aios_b200."""
    from oracle import reference_run

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    mods = reference_run.install()
    llm = reference_run.build_llm(mods, reference_run.SHAPES["S10"], num_pages=256 * 16)
    engine = mods.ime.ImeCompletionEngine(llm)
    kc = mods.ime.ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                                      max_new_tokens=12, temperature=0.8, top_k=50, top_p=0.9, seed=0)
    texts = prefixes(llm.tokenizer, llm.config.vocab_size, warmup + keystrokes, seed=seed)
    times = []
    for i, text in enumerate(texts):
        engine.reset_prefix_cache()
        t0 = time.perf_counter()
        engine.complete(text, kc)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": len(times) / total, "unit": "keystrokes/s", "cores": threads, "kind": "reference",
            "p50_ms": statistics.median(times) * 1e3, "p95_ms": percentile(times, 0.95) * 1e3,
            "sample": f"{len(times)} keystrokes of the bench workload through the unmodified reference "
                      f"ImeCompletionEngine.complete (fp32, {threads} threads, CPU shims for FlashInfer and "
                      f"the KV buffer), {total:.1f} s"}


def run_port(keystrokes: int, warmup: int) -> dict:
    """Fallback of the reference arm when no reference install is present: the
    oracle restatement of the same keystroke (fp32, all host threads)."""
    from aios_b200.models import shapes
    from aios_b200.models.minimind_ime import MiniMindIMEForCausalLM
    from aios_b200.models.weight import synthetic_state_dict
    from aios_b200.tokenizer import SyntheticTokenizer
    from oracle.engine import OracleEngine
    from oracle.model import OracleModel

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = shapes.S10
    with torch.device("meta"):
        meta = MiniMindIMEForCausalLM(cfg)
    model = OracleModel(cfg, synthetic_state_dict(meta, seed=0), dtype=torch.float32, num_slots=256 * 16)
    tok = SyntheticTokenizer(cfg.vocab_size)
    eng = OracleEngine(model, tok, num_pages=256, page_size=16)
    kc = keystroke_config()
    texts = prefixes(tok, cfg.vocab_size, warmup + keystrokes, seed=1234)
    times = []
    for i, text in enumerate(texts):
        ids = [1, *tok.encode(text)]
        eng.reset_prefix()
        t0 = time.perf_counter()
        logits, _, _ = eng.prepare_prefix(ids, kc.max_sampling_attempts)
        tr = eng.run_round(prefix_logits=logits, prefix_len=len(ids), row_offset=0, attempts=8,
                           max_new_tokens=kc.max_new_tokens, min_new_tokens=kc.min_new_tokens, seed=kc.seed,
                           temperature=kc.temperature, top_k=kc.top_k, top_p=kc.top_p)
        eng.release(tr.allocated)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": len(times) / total, "unit": "keystrokes/s", "cores": threads, "kind": "port",
            "p50_ms": statistics.median(times) * 1e3, "p95_ms": percentile(times, 0.95) * 1e3,
            "sample": f"{len(times)} keystrokes of the bench workload (fp32, oracle restatement, "
                      f"{threads} threads), {total:.1f} s"}


def reference_subprocess(keystrokes: int) -> dict | None:
    """The reference arm in a child process (keeps the reference's import-time
    shims out of the GPU process); returns its cpu_baseline, or None."""
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", str(keystrokes),
           "--warmup", "3"]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    for line in reversed(proc.stdout.splitlines()):
        if line.startswith("{"):
            return json.loads(line).get("cpu_baseline")
    return None


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
# dram__bytes_read.sum + dram__bytes_write.sum summed over the 57 linear launches
# of one decode step, from one ncu capture of the `linears` NVTX range below with
# `--cache-control none`, so that L2 carries over between launches and replays as
# it does in the timed loop. It is
# below the 201,326,592 algorithmic bytes: with cache-streaming weight loads,
# about 15% of the weights are still in L2 when the next replay reads them.
# Captured again after the linears gained the early-successor flag and the
# explicit launch bounds (171,439,616 B read + 322,816 B written).
DECODE_LINEAR_TRAFFIC = 171_762_432
# The same for one launch of the persistent decode-step kernel (None until an ncu
# capture of it exists).
DECODE_STEP_TRAFFIC = None


def pin_rank_cores(local_rank: int, local_world: int) -> list[int]:
    """Pins this rank's process to its own contiguous share of the host cores it
    may use (each replica's launch loop then runs without sharing cores with the
    others); returns the cores."""
    cores = sorted(os.sched_getaffinity(0))
    share = max(1, len(cores) // max(1, local_world))
    mine = cores[local_rank * share : (local_rank + 1) * share] or cores
    os.sched_setaffinity(0, mine)
    return mine


def max_over_ranks(values: list[float], world: int, device=None) -> list[float]:
    """Each timing's maximum over all ranks (one all-reduce of host values over
    the gloo group: the replicas exchange nothing on the GPU); unchanged for one
    rank. The slowest replica bounds the job."""
    t = torch.tensor(values, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def gather_over_ranks(value: float, world: int) -> list[float]:
    """Every rank's value, in rank order (host-side gather over gloo)."""
    if world <= 1:
        return [value]
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64)
    out = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x) for x in out]


def replica_throughput(world: int, steps: int, device_ms: float) -> float:
    """Whole-job keystrokes/s: every replica runs `steps` keystrokes, and
    `device_ms` is the slowest replica's timed region."""
    return world * steps / (device_ms * 1e-3)


def decode_linear_roofline(llm, peaks: dict) -> dict:
    """Times the linear launches of one decode step (8 rows: 14 x
    {qkv, o, gate_up+SwiGLU, down} + LM head, the same shapes and weights as the
    keystroke) as a captured graph, with CUDA events on the launching stream."""
    from aios_b200 import _lib
    from aios_b200.kernel import ops

    dev = llm.device
    cfg = llm.config
    rows = 8
    layers = llm.model.model.layers.op_list
    xo = torch.randn(rows, cfg.num_qo_heads * cfg.head_dim, device=dev).to(torch.bfloat16)
    xf = torch.randn(rows, cfg.intermediate_size, device=dev).to(torch.bfloat16)
    res = torch.randn(rows, cfg.hidden_size, device=dev).to(torch.bfloat16)
    stats = ops.RowStats(torch.randn(rows, cfg.hidden_size, device=dev),
                         torch.rand(cfg.hidden_size // 128, rows, device=dev) * 100)
    nw = torch.ones(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    outs = {}

    def run():
        # the model's decode GEMMs: norm-from-statistics qkv / gate_up / LM head,
        # residual-add + statistics o / down
        for i, layer in enumerate(layers):
            a, m = layer.self_attn, layer.mlp
            outs["qkv"] = ops.linear_stat_norm(stats, nw, 1e-6, a.qkv_proj.weight)
            outs["o"] = ops.linear_add_stat(xo, a.o_proj.weight, res)
            outs["gu"] = ops.linear_stat_norm(stats, nw, 1e-6, m.gate_up_proj.packed_weight(),
                                              epilogue=_lib.EPI_SILU_MUL)
            outs["d"] = ops.linear_add_stat(xf, m.down_proj.weight, res)
        outs["lm"] = ops.linear_stat_norm(stats, nw, 1e-6, llm.model.model.embed_tokens.weight)

    run()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    for _ in range(3):
        g.replay()
    iters = 50
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    start.record(stream)
    for _ in range(iters):
        g.replay()
    end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / iters
    # one extra replay in its own NVTX range: the launches an ncu traffic capture selects
    torch.cuda.nvtx.range_push("linears")
    g.replay()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    launches = 4 * len(layers) + 1
    wbytes = sum(layer.self_attn.qkv_proj.weight.numel() + layer.self_attn.o_proj.weight.numel()
                 + layer.mlp.gate_up_proj.weight.numel() + layer.mlp.down_proj.weight.numel() for layer in layers)
    wbytes = 2 * (wbytes + llm.model.model.embed_tokens.weight.numel())
    achieved = wbytes / (ms * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    return {"bound": "hbm", "kernel": "gemv_mma_kernel (decode linears, 8 rows, register-operand MMA)", "achieved": round(achieved, 1),
            "peak": peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": DECODE_LINEAR_TRAFFIC,
            "traffic_unit": "bytes per decode step (57 launches)",
            "traffic_source": "one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum, --cache-control none) "
                              "of the `linears` NVTX range of this function, on the current gemv_mma_kernel",
            "algorithmic_bytes_per_step": wbytes,
            "launches_per_step": launches, "us_per_step": round(ms * 1e3, 2),
            "us_per_launch": round(ms * 1e3 / launches, 3)}


PREFILL_GEMM_ROWS = (13, 32, 64, 128, 512, 2048)
GEMV_MAX_ROWS = int(os.environ.get("AIOSB_GEMV_MAX_ROWS", "512"))  # the library's dispatch bound


def prefill_gemm_sweep(llm, peaks: dict) -> dict:
    """The linears of one S10 forward (14 x {qkv, o + residual add, gate_up +
    SwiGLU, down + residual add}) at M token rows, M in {13, 128, 512, 2048}:
    a keystroke prefix through a long prompt. Each pass reads all 176 MB of layer
    weights (more than L2). Rows <= 16 run the register-operand MMA GEMV, more
    rows the tcgen05 GEMM. Timed as a captured graph with CUDA events on the
    launching stream; FLOPs = 2 x M x (weight elements). The kernel that ran is
    named per M (the GEMV takes up to 512 rows, as 16-row groups above 16)."""
    from aios_b200 import _lib
    from aios_b200.kernel import ops

    dev = llm.device
    cfg = llm.config
    layers = llm.model.model.layers.op_list
    welems = sum(l.self_attn.qkv_proj.weight.numel() + l.self_attn.o_proj.weight.numel()
                 + l.mlp.gate_up_proj.weight.numel() + l.mlp.down_proj.weight.numel() for l in layers)
    peak = peaks.get("bf16_tflops", BF16_FALLBACK_TFLOPS)
    out = {"peak_tflops": peak, "peak_source": "measured (burst)" if "bf16_tflops" in peaks else "fallback",
           "weight_bytes": 2 * welems, "rows": {}}
    stream = torch.cuda.current_stream(dev)
    for m in PREFILL_GEMM_ROWS:
        g = torch.Generator(device=dev).manual_seed(m)
        x = (torch.randn(m, cfg.hidden_size, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        xo = (torch.randn(m, cfg.num_qo_heads * cfg.head_dim, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        xf = (torch.randn(m, cfg.intermediate_size, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        res = torch.zeros(m, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        qkv = torch.empty(m, layers[0].self_attn.qkv_proj.weight.shape[0], dtype=torch.bfloat16, device=dev)
        act = torch.empty(m, cfg.intermediate_size, dtype=torch.bfloat16, device=dev)

        def run():
            for layer in layers:
                a, mlp = layer.self_attn, layer.mlp
                ops.linear(x, a.qkv_proj.weight, out=qkv)
                ops.linear(xo, a.o_proj.weight, out=res, epilogue=_lib.EPI_ADD, residual=res)
                ops.linear(x, mlp.gate_up_proj.packed_weight(), out=act, epilogue=_lib.EPI_SILU_MUL)
                ops.linear(xf, mlp.down_proj.weight, out=res, epilogue=_lib.EPI_ADD, residual=res)

        run()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run()
        for _ in range(2):
            graph.replay()
        iters = 10
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        start.record(stream)
        for _ in range(iters):
            graph.replay()
        end.record(stream)
        end.synchronize()
        ms = start.elapsed_time(end) / iters
        tflops = 2.0 * m * welems / (ms * 1e-3) / 1e12
        out["rows"][str(m)] = {"kernel": "gemv_mma_kernel" if m <= GEMV_MAX_ROWS else "gemm_tc_kernel",
                               "us_per_forward": round(ms * 1e3, 2), "us_per_linear": round(ms * 1e3 / (4 * len(layers)), 2),
                               "tflops": round(tflops, 1), "frac_of_bf16_peak": round(tflops / peak, 4),
                               "weight_gbs": round(2 * welems / (ms * 1e-3) / 1e9, 1)}
        del graph
    ops.check_status(dev)
    return out


def decode_forward_roofline(engine, llm, peaks: dict) -> dict:
    """The default decode forward (the chain of per-kernel launches the step graphs
    replay, without the group step) of `llm` at 8 active rows on the first decode
    position after the last keystroke's prefix (its prefix KV and page-table rows
    are real), captured 5 times per graph and timed with CUDA events on the
    launching stream. Algorithmic bytes: every weight once (the tied LM head once)
    plus the attention's K/V reads and its q / o rows."""
    from aios_b200.kernel import ops
    from aios_b200.runtime.group import stage_class

    rt = engine._runtime
    dev = llm.device
    cfg = llm.config
    rows = 8
    p_len = len(engine._prefix_slots)
    kv = llm.mha_kv_cache
    rt.active[:rows].fill_(1)
    rt.positions[:rows].fill_(p_len)
    rt.seq_lens[:rows].fill_(p_len + 1)
    rt.row_table[:rows].copy_(torch.arange(rows, dtype=torch.int32, device=dev))
    rt.prefix_len_view.fill_(p_len)
    spare = torch.arange(kv.num_slots - rows, kv.num_slots, dtype=torch.int32, device=dev)  # unused pool tail
    rt.out_loc[:rows].copy_(spare)
    llm.ctx.page_table[:rows, p_len].copy_(spare)
    rt.tokens[:rows].copy_(torch.arange(100, 100 + rows, dtype=torch.int32, device=dev))
    batch = rt._decode_batch(rows, stage_class(p_len))

    def forward():
        with llm.ctx.forward_batch(batch):
            llm.model.forward()

    forward()
    torch.cuda.synchronize(dev)
    per_graph = 5
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(per_graph):
            forward()
    g.replay()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    start.record(stream)
    for _ in range(reps):
        g.replay()
    end.record(stream)
    end.synchronize()
    us = start.elapsed_time(end) / (reps * per_graph) * 1e3
    del g
    ops.check_status(dev)
    rt.active.zero_()
    layers = llm.model.model.layers.op_list
    wbytes = sum(layer.self_attn.qkv_proj.weight.numel() + layer.self_attn.o_proj.weight.numel()
                 + layer.mlp.gate_up_proj.weight.numel() + layer.mlp.down_proj.weight.numel() for layer in layers)
    wbytes = 2 * (wbytes + llm.model.model.embed_tokens.weight.numel())
    hkv, hd, hq = cfg.num_kv_heads, cfg.head_dim, cfg.num_qo_heads
    attn_bytes = len(layers) * (p_len * hkv * hd * 2 * 2 + rows * hkv * hd * 2 * 2 + 2 * rows * hq * hd * 2)
    total = wbytes + attn_bytes
    achieved = total / (us * 1e-6) / 1e9
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    return {"bound": "hbm", "us_per_step": round(us, 2), "algorithmic_bytes_per_step": total,
            "weight_bytes": wbytes, "achieved_gbs": round(achieved, 1), "peak": peak,
            "frac": round(achieved / peak, 4), "layers": len(layers), "prefix_tokens": p_len}


def decode_step_roofline(engine, llm, peaks: dict) -> dict:
    """Times the persistent decode-step kernel alone (CUDA events on the launching
    stream, a graph of back-to-back launches): one decode forward of the bench
    group, 8 active rows at the first decode position after the 13-token prefix of
    the last keystroke (so its prefix KV and page-table rows are real). Algorithmic
    bytes per launch: every weight once (201,326,592 B for S10) plus the
    attention's K/V reads (the prefix once per KV head, each row's suffix) and its
    q / o rows (the cascade formula)."""
    from aios_b200 import _lib

    rt = engine._runtime
    was_on = rt._step_plan is not None
    if not rt.use_persistent_step():
        return decode_linear_roofline(llm, peaks)
    plan = rt._step_plan
    dev = llm.device
    cfg = llm.config
    rows = 8
    prefix = engine._prefix_slots
    p_len = len(prefix)
    kv = llm.mha_kv_cache
    rt.active[:rows].fill_(1)
    rt.positions[:rows].fill_(p_len)
    rt.seq_lens[:rows].fill_(p_len + 1)
    rt.row_table[:rows].copy_(torch.arange(rows, dtype=torch.int32, device=dev))
    rt.prefix_len_view.fill_(p_len)
    spare = torch.arange(kv.num_slots - rows, kv.num_slots, dtype=torch.int32, device=dev)  # unused pool tail
    rt.out_loc[:rows].copy_(spare)
    llm.ctx.page_table[:rows, p_len].copy_(spare)
    rt.tokens[:rows].copy_(torch.arange(100, 100 + rows, dtype=torch.int32, device=dev))
    args = _lib.DecodeStepArgs.from_buffer_copy(plan["args"])
    args.rows = rows
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        _lib.call("aiosb_decode_step", ctypes.byref(args), stream.cuda_stream)
    torch.cuda.synchronize(dev)
    per_graph = 10
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(per_graph):
            _lib.call("aiosb_decode_step", ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream)
    g.replay()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    start.record(stream)
    for _ in range(reps):
        g.replay()
    end.record(stream)
    end.synchronize()
    us = start.elapsed_time(end) / (reps * per_graph) * 1e3
    # one extra launch in its own NVTX range: the one an ncu traffic capture selects
    torch.cuda.nvtx.range_push("decode_step")
    _lib.call("aiosb_decode_step", ctypes.byref(args), stream.cuda_stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    from aios_b200.kernel import ops

    ops.check_status(dev)
    rt.active.zero_()
    rt.use_persistent_step(was_on)
    layers = llm.model.model.layers.op_list
    wbytes = sum(layer.self_attn.qkv_proj.weight.numel() + layer.self_attn.o_proj.weight.numel()
                 + layer.mlp.gate_up_proj.weight.numel() + layer.mlp.down_proj.weight.numel() for layer in layers)
    wbytes = 2 * (wbytes + llm.model.model.embed_tokens.weight.numel())
    hkv, hd, hq = cfg.num_kv_heads, cfg.head_dim, cfg.num_qo_heads
    attn_bytes = len(layers) * (p_len * hkv * hd * 2 * 2 + rows * 1 * hkv * hd * 2 * 2 + 2 * rows * hq * hd * 2)
    total = wbytes + attn_bytes
    achieved = total / (us * 1e-6) / 1e9
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    return {"bound": "hbm", "kernel": "decode_step_kernel (persistent decode forward, 8 rows, one launch per step)",
            "achieved": round(achieved, 1), "peak": peak,
            "peak_source": "measured (burst copy)" if "hbm_gbs" in peaks else "fallback", "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": DECODE_STEP_TRAFFIC,
            "traffic_unit": "bytes per launch (dram read + write, ncu)",
            "algorithmic_bytes_per_launch": total, "weight_bytes": wbytes, "attention_bytes": attn_bytes,
            "us_per_launch": round(us, 2), "launches_timed": reps * per_graph}


def mixer_chain(dev) -> dict:
    """BASELINE config 1 on the GPU: 65-mixer chain (banks of depth 1..9 + partial,
    [8, 768] bf16) and a bandwidth point at 32768 rows (sources >> L2)."""
    from aios_b200.kernel import ops

    g = torch.Generator(device=dev).manual_seed(0)
    banks = [torch.randn(d, 8, 768, generator=g, device=dev).to(torch.bfloat16) for d in range(1, 10)]
    partial = torch.randn(8, 768, generator=g, device=dev).to(torch.bfloat16)
    wq = [torch.randn(768, generator=g, device=dev) * 0.02 for _ in range(65)]
    out = torch.empty(8, 768, dtype=torch.bfloat16, device=dev)

    def chain():
        i = 0
        for b in range(8):
            for layer in range(4):
                ops.b200_attnres_mix(banks[b], None if layer == 0 else partial, wq[i], 1e-6, output_buffer=out)
                ops.b200_attnres_mix(banks[b], partial, wq[i + 1], 1e-6, output_buffer=out)
                i += 2
        ops.b200_attnres_mix(banks[8], None, wq[64], 1e-6, output_buffer=out)

    chain()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for _ in range(3):
        graph.replay()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(20):
        graph.replay()
    e.record()
    e.synchronize()
    chain_us = s.elapsed_time(e) / 20 * 1e3
    chain_bytes = 0
    for b in range(8):
        d = b + 1
        chain_bytes += (d * 8 * 768 * 2 + 8 * 768 * 2 + 768 * 4)  # layer 0 of the block: no partial
        chain_bytes += 7 * ((d + 1) * 8 * 768 * 2 + 8 * 768 * 2 + 768 * 4)
    chain_bytes += 9 * 8 * 768 * 2 + 8 * 768 * 2 + 768 * 4
    n = 32768
    big = torch.randn(8, n, 768, generator=g, device=dev).to(torch.bfloat16)
    bp = torch.randn(n, 768, generator=g, device=dev).to(torch.bfloat16)
    bo = torch.empty(n, 768, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        ops.b200_attnres_mix(big, bp, wq[0], 1e-6, output_buffer=bo)
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(20):
        ops.b200_attnres_mix(big, bp, wq[0], 1e-6, output_buffer=bo)
    e.record()
    e.synchronize()
    big_ms = s.elapsed_time(e) / 20
    big_bytes = 9 * n * 768 * 2 + n * 768 * 2 + 768 * 4
    del big, bp, bo
    # bandwidth sweep over token counts: 8 bank sources + the partial, [N, 768]
    sweep = {}
    for n in (8, 64, 512, 4096, 32768, 131072):
        sb = torch.randn(8, n, 768, generator=g, device=dev).to(torch.bfloat16)
        sp = torch.randn(n, 768, generator=g, device=dev).to(torch.bfloat16)
        so = torch.empty(n, 768, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            ops.b200_attnres_mix(sb, sp, wq[0], 1e-6, output_buffer=so)
        iters = 20 if n >= 4096 else 100
        torch.cuda.synchronize(dev)
        s.record()
        for _ in range(iters):
            ops.b200_attnres_mix(sb, sp, wq[0], 1e-6, output_buffer=so)
        e.record()
        e.synchronize()
        us = s.elapsed_time(e) / iters * 1e3
        sweep[str(n)] = {"us": round(us, 2), "gbs": round((10 * n * 768 * 2 + 768 * 4) / (us * 1e-6) / 1e9, 1)}
        del sb, sp, so
    return {"chain65_us": round(chain_us, 2), "chain65_gbs": round(chain_bytes / (chain_us * 1e-6) / 1e9, 1),
            "n32768_gbs": round(big_bytes / (big_ms * 1e-3) / 1e9, 1), "sweep_9src": sweep}


def stream_texts(tokenizer, vocab: int, seed: int, keystrokes: int = 40) -> tuple[list[str], int]:
    """a seeded typing stream. Every keystroke appends 1-2
    random tokens to the previous prefix, except 10% backspaces that drop the
    last token (which the engine answers with a full re-prefill)."""
    import random

    rng = random.Random(seed)
    ids = [rng.randint(10, vocab - 1) for _ in range(2)]
    texts, backspaces = [], 0
    for _ in range(keystrokes):
        if rng.random() < 0.1 and len(ids) > 1:
            ids = ids[:-1]
            backspaces += 1
        else:
            ids = ids + [rng.randint(10, vocab - 1) for _ in range(rng.randint(1, 2))]
        texts.append(tokenizer.text_for(ids))
    return texts, backspaces


def keystroke_stream(engine, llm, seed: int) -> dict:
    """Config 5 on one GPU, through ``complete``: the 40-keystroke stream with
    token-LCP reuse of the prefix KV, run once to warm the prefill graphs and
    once timed (keystrokes in sequence, as with a 30-150 ms think time); then the
    forced-overlap variant, where every next keystroke arrives 2 ms after the
    previous one started, so latest-wins cancels the group in flight."""
    from concurrent.futures import ThreadPoolExecutor

    cfg = keystroke_config()
    texts, backspaces = stream_texts(llm.tokenizer, llm.config.vocab_size, seed)
    out = {"keystrokes": len(texts), "backspaces": backspaces}
    for _ in range(2):
        engine.reset_prefix_cache()
        res = [engine.complete(t, cfg) for t in texts]
    lat = [r.latency_ms for r in res]
    out.update(p50_ms=round(statistics.median(lat), 3), p95_ms=round(percentile(lat, 0.95), 3),
               gpu_p50_ms=round(statistics.median([r.gpu_latency_ms for r in res]), 3),
               reused_prefix_tokens=sum(r.reused_prefix_tokens for r in res))
    engine.reset_prefix_cache()
    device = llm.device

    def complete_on_device(text, token):
        torch.cuda.set_device(device)
        return engine.complete(text, cfg, token)

    with ThreadPoolExecutor(max_workers=4) as pool:
        futures = []
        for t in texts:
            token = engine.new_generation()  # cancels the keystroke in flight
            futures.append((time.perf_counter(), pool.submit(complete_on_device, t, token)))
            time.sleep(0.002)
        done = []
        for t0, fut in futures:
            r = fut.result()
            done.append((r, (time.perf_counter() - t0) * 1e3))
    final = done[-1]
    out["overlap"] = {"arrival_gap_ms": 2.0, "cancelled": sum(r.cancelled for r, _ in done),
                      "completed": sum(not r.cancelled for r, _ in done),
                      "last_keystroke_ms": round(final[1], 3), "last_cancelled": final[0].cancelled}
    return out


def _latencies(engine, texts: list[str], cfg, warmup: int) -> list:
    results = []
    for i, text in enumerate(texts):
        engine.reset_prefix_cache()
        r = engine.complete(text, cfg)
        if i >= warmup:
            results.append(r)
    return results


def shape_keystroke(shape: str, dev, keystrokes: int = 20, warmup: int = 5) -> dict:
    """The bench keystroke ([BOS]+12, 8 candidates x 12 tokens, T 0.8, top-k 50,
    top-p 0.9, 16-token pages x 256) on another model shape, through ``complete``:
    S06 is BASELINE config 2 (8 layers, 8 q / 2 kv heads of 96, vocab 6400), S10L
    the same dims at 14 layers."""
    from aios_b200 import ImeCompletionEngine, LLM
    from aios_b200.models import shapes

    llm_s = LLM(config=getattr(shapes, shape), seed=0, page_size=16, num_pages=256, device=str(dev))
    eng_s = ImeCompletionEngine(llm_s)
    res = _latencies(eng_s, prefixes(llm_s.tokenizer, llm_s.config.vocab_size, warmup + keystrokes, seed=606),
                     keystroke_config(), warmup)
    lat = [r.latency_ms for r in res]
    out = {"p50_ms": round(statistics.median(lat), 3), "p95_ms": round(percentile(lat, 0.95), 3),
           "gpu_p50_ms": round(statistics.median([r.gpu_latency_ms for r in res]), 3),
           "decode_tok_s": round(sum(r.generated_tokens for r in res) / (sum(r.gpu_latency_ms for r in res) * 1e-3), 1),
           "layers": llm_s.config.num_layers, "head_dim": llm_s.config.head_dim, "vocab": llm_s.config.vocab_size}
    del eng_s, llm_s
    torch.cuda.empty_cache()
    return out


HISTORY_PREFIXES = (13, 32, 128, 256, 448)


def decode_history_crossover(engine, llm) -> dict:
    """The S10 bench keystroke (8 candidates x 12 tokens) at prefixes of 13 to 448
    tokens (the 512-position context), with each way the decode attention can
    read the key history: per-row staging, prefix-once cluster staging, and the
    cluster-cascade kernel. p50 over 8 keystrokes after 2 warm-up ones; the
    runtime's default mode is restored afterwards."""
    rt = engine._runtime
    default = rt.history_mode
    out = {}
    for n in HISTORY_PREFIXES:
        texts = prefixes(llm.tokenizer, llm.config.vocab_size, 10, seed=500 + n, length=n - 1)
        row = {}
        for mode in ("staged", "prefix_once", "cascade"):
            rt.use_history_mode(mode)
            lat = [r.latency_ms for r in _latencies(engine, texts, keystroke_config(), 2)]
            row[mode] = round(statistics.median(lat), 3)
        out[str(n)] = row
    from aios_b200.runtime.group import HISTORY_MODES

    rt.use_history_mode(next(k for k, v in HISTORY_MODES.items() if v == default))
    return out


def config_sweeps(engine, llm, dev) -> dict:
    """BASELINE configs 2, 3 and 4 through ``complete``.
    Config 2: the bench keystroke on S06 (and on S10L, S06's dims at 14 layers).
    Config 3: the S10 keystroke at prefix lengths 4/8/16/32 after [BOS], 8
    candidates x 16 tokens. Config 4: the S21 Block-AttnRes model (32 layers, 8
    blocks, 65 mixers per forward), a 16-token prefix and refill rounds of 8 up to
    24 candidates, each round freeing the previous round's suffix KV (a 2-character
    candidate limit makes every candidate invalid, so the refill always runs to
    the 24-attempt budget)."""
    from aios_b200 import ImeCompletionEngine, ImeGenerationConfig, LLM
    from aios_b200.models import shapes

    out = {"s10_prefix_sweep": {}}
    cfg3 = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=8, refill_batch_size=8,
                               max_new_tokens=16, temperature=0.8, top_k=50, top_p=0.9, seed=0)
    for n in (4, 8, 16, 32):
        res = _latencies(engine, prefixes(llm.tokenizer, llm.config.vocab_size, 13, seed=77 + n, length=n), cfg3, 3)
        lat = [r.latency_ms for r in res]
        out["s10_prefix_sweep"][str(n)] = {"p50_ms": round(statistics.median(lat), 3),
                                           "p95_ms": round(percentile(lat, 0.95), 3)}
    out["decode_history"] = decode_history_crossover(engine, llm)
    # the decode forward after one bench keystroke ([BOS]+12 prefix)
    _latencies(engine, prefixes(llm.tokenizer, llm.config.vocab_size, 1, seed=1234), keystroke_config(), 0)
    out["s10_decode_forward"] = decode_forward_roofline(engine, llm, measured_peaks())
    # the other shapes build their own LLM (each takes over the process-global
    # context), so they run after every keystroke of the S10 engine
    out["s06_keystroke"] = shape_keystroke("S06", dev)
    out["s10l_keystroke"] = shape_keystroke("S10L", dev)
    llm21 = LLM(config=shapes.S21, seed=0, page_size=16, num_pages=256, device=str(dev))
    eng21 = ImeCompletionEngine(llm21)
    cfg4 = ImeGenerationConfig(sampling_attempts=8, max_sampling_attempts=24, refill_batch_size=8,
                               max_new_tokens=16, temperature=0.8, top_k=50, top_p=0.9, max_candidate_chars=2, seed=0)
    res = _latencies(eng21, prefixes(llm21.tokenizer, llm21.config.vocab_size, 10, seed=21, length=16), cfg4, 2)
    lat = [r.latency_ms for r in res]
    out["s21_refill"] = {"p50_ms": round(statistics.median(lat), 3), "p95_ms": round(percentile(lat, 0.95), 3),
                         "attempts": res[0].sampling_attempts, "refill_rounds": res[0].refill_rounds,
                         "decode_tok_s": round(sum(r.generated_tokens for r in res) / (sum(r.gpu_latency_ms for r in res) * 1e-3), 1),
                         "decode_forward": decode_forward_roofline(eng21, llm21, measured_peaks())}
    del eng21, llm21
    torch.cuda.empty_cache()
    return out


def run_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch.distributed as dist

    from aios_b200 import ImeCompletionEngine, LLM, _lib
    from aios_b200.kernel import ops
    from aios_b200.models import shapes

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=256, device=f"cuda:{local_rank}")
    engine = ImeCompletionEngine(llm)
    cfg = keystroke_config()
    texts = prefixes(llm.tokenizer, llm.config.vocab_size, args.warmup + args.steps, seed=1234 + rank)
    for text in texts[: args.warmup]:
        engine.reset_prefix_cache()
        engine.complete(text, cfg)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    rt = engine._runtime
    pr = engine._prefix_runner
    h2d0 = rt.h2d_bytes + pr.h2d_bytes + ops.transfer_bytes["h2d"]
    d2h0 = rt.d2h_bytes + ops.transfer_bytes["d2h"]
    launches0 = _lib.launches
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    # one sampler per rank: every 50 ms on one GPU, every 200 ms with more ranks
    # (eight samplers at 50 ms would compete with the ranks' launch loops)
    with ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else 0,
                      50 if world == 1 else 200) as clocks:
        torch.cuda.synchronize(dev)
        clocks.mark()
        wall0 = time.perf_counter()
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        for text in texts[args.warmup :]:
            engine.reset_prefix_cache()
            results.append(engine.complete(text, cfg))
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        end.synchronize()
        wall = time.perf_counter() - wall0
    device_ms = start.elapsed_time(end)
    launches = _lib.launches - launches0
    h2d = (rt.h2d_bytes + pr.h2d_bytes + ops.transfer_bytes["h2d"] - h2d0) / args.steps
    d2h = (rt.d2h_bytes + ops.transfer_bytes["d2h"] - d2h0) / args.steps
    per_rank_ms = gather_over_ranks(device_ms / args.steps, world)
    device_ms, wall = max_over_ranks([device_ms, wall], world, dev)
    if rank != 0:
        return None
    peaks = measured_peaks()
    roof = None if args.no_extras else decode_linear_roofline(llm, peaks)
    step_kernel = None if args.no_extras else decode_step_roofline(engine, llm, peaks)
    prefill_gemm = None if args.no_extras else prefill_gemm_sweep(llm, peaks)
    mixer = None if args.no_extras else mixer_chain(dev)
    kstream = None if args.no_extras else keystroke_stream(engine, llm, seed=4321 + rank)
    sweeps = None if args.no_extras else config_sweeps(engine, llm, dev)
    lat = [r.latency_ms for r in results]
    gpu_lat = [r.gpu_latency_ms for r in results]
    gen = sum(r.generated_tokens for r in results)
    active = sum(r.active_model_tokens for r in results)
    line = {
        "metric": "Top-3 keystroke latency p50/p95 ms (8 cand), decode tok/s, mixer HBM GB/s",
        "value": round(replica_throughput(world, args.steps, device_ms), 3),
        "unit": "keystrokes/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(device_ms / args.steps, 4),
        "per_rank_ms_per_step": [round(x, 4) for x in per_rank_ms],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random weights, seeded prefixes, synthetic tokenizer)",
        "config": bench_config(world),
        "latency_ms": {"p50": round(statistics.median(lat), 3), "p95": round(percentile(lat, 0.95), 3),
                       "gpu_p50": round(statistics.median(gpu_lat), 3),
                       "gpu_p95": round(percentile(gpu_lat, 0.95), 3)},
        "decode_tok_s": round(world * gen / (device_ms * 1e-3), 1),
        "active_model_tok_s": round(active / (sum(gpu_lat) * 1e-3), 1),
        "mixer": mixer,
        "stream": kstream,
        "configs": sweeps,
        "e2e": {"value": round(world * args.steps / wall, 3), "unit": "keystrokes/s",
                "h2d_bytes_per_step": int(round(h2d)), "d2h_bytes_per_step": int(round(d2h))},
        "gpu_launches": launches,
        "roofline": roof,
        "persistent_step": step_kernel,
        "prefill_gemm": prefill_gemm,
        "clocks": clocks.summary(),
    }
    return line


def kernel_case(name: str) -> None:
    """Small single-kernel workloads for full ncu captures (1 GPU, a few GB).
    linears: the decode linears of every S10 layer in order, 8 rows, eagerly
    (the 176 MB of layer weights exceed L2, so each launch reads DRAM);
    decode_step: two bench keystrokes (the persistent decode-step kernel, 11
    launches each, 201 MB of weights per launch);
    mixer: the AttnRes mixer on 32768 tokens of 8 bank sources + partial
    (the stream kernel; 504 MB of traffic per launch)."""
    from aios_b200 import LLM, _lib
    from aios_b200.kernel import ops
    from aios_b200.models import shapes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if name == "linears":
        llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=16, device="cuda:0")
        cfg = llm.config
        rows = 8
        xo = torch.randn(rows, cfg.num_qo_heads * cfg.head_dim, device=dev).to(torch.bfloat16)
        xf = torch.randn(rows, cfg.intermediate_size, device=dev).to(torch.bfloat16)
        res = torch.randn(rows, cfg.hidden_size, device=dev).to(torch.bfloat16)
        stats = ops.RowStats(torch.randn(rows, cfg.hidden_size, device=dev),
                             torch.rand(cfg.hidden_size // 128, rows, device=dev) * 100)
        nw = torch.ones(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        for _ in range(2):
            for layer in llm.model.model.layers.op_list:
                a, m = layer.self_attn, layer.mlp
                ops.linear_stat_norm(stats, nw, 1e-6, a.qkv_proj.weight)
                ops.linear_add_stat(xo, a.o_proj.weight, res)
                ops.linear_stat_norm(stats, nw, 1e-6, m.gate_up_proj.packed_weight(), epilogue=_lib.EPI_SILU_MUL)
                ops.linear_add_stat(xf, m.down_proj.weight, res)
    elif name == "decode_step":
        # two bench keystrokes: 11 persistent decode-step launches each (S10, 8 rows)
        from aios_b200 import ImeCompletionEngine

        llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=256, device="cuda:0")
        engine = ImeCompletionEngine(llm)
        for text in prefixes(llm.tokenizer, llm.config.vocab_size, 2, seed=1234):
            engine.reset_prefix_cache()
            engine.complete(text, keystroke_config())
    elif name.startswith("gemm_m"):
        # one S10 layer's four linears at M token rows, eagerly, three times over
        # the same weights (the 12.6 MB of one layer stay in L2 after the first)
        from aios_b200 import _lib

        m = int(name[len("gemm_m"):])
        llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=16, device="cuda:0")
        cfg = llm.config
        layer = llm.model.model.layers.op_list[0]
        a, mlp = layer.self_attn, layer.mlp
        x = (torch.randn(m, cfg.hidden_size, device=dev) * 0.5).to(torch.bfloat16)
        xf = (torch.randn(m, cfg.intermediate_size, device=dev) * 0.5).to(torch.bfloat16)
        res = torch.zeros(m, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            ops.linear(x, a.qkv_proj.weight)
            ops.linear(x, a.o_proj.weight, out=res, epilogue=_lib.EPI_ADD, residual=res)
            ops.linear(x, mlp.gate_up_proj.packed_weight(), epilogue=_lib.EPI_SILU_MUL)
            ops.linear(xf, mlp.down_proj.weight, out=res, epilogue=_lib.EPI_ADD, residual=res)
    elif name.startswith("prefill_attn_t"):
        # S10 keystrokes whose prefix is T tokens ([BOS] + T - 1 characters): the
        # prefix prefill runs the one-launch attention (T <= 64) or the two-kernel
        # path (longer), 14 layers per keystroke
        from aios_b200 import ImeCompletionEngine

        t = int(name[len("prefill_attn_t"):])
        llm = LLM(config=shapes.S10, seed=0, page_size=16, num_pages=256, device="cuda:0")
        engine = ImeCompletionEngine(llm)
        for text in prefixes(llm.tokenizer, llm.config.vocab_size, 2, seed=1234, length=t - 1):
            engine.reset_prefix_cache()
            engine.complete(text, keystroke_config())
    elif name == "mixer":
        g = torch.Generator(device=dev).manual_seed(0)
        bank = torch.randn(8, 32768, 768, generator=g, device=dev).to(torch.bfloat16)
        part = torch.randn(32768, 768, generator=g, device=dev).to(torch.bfloat16)
        wq = torch.randn(768, generator=g, device=dev) * 0.02
        out = torch.empty(32768, 768, dtype=torch.bfloat16, device=dev)
        for _ in range(4):
            ops.b200_attnres_mix(bank, part, wq, 1e-6, output_buffer=out)
    else:
        raise SystemExit(f"unknown kernel case {name}")
    torch.cuda.synchronize(dev)
    ops.check_status(dev)
    print(f"kernel case {name}: ok")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-sample", type=int, default=15, help="keystrokes timed for the CPU baseline (0: skip)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the roofline / mixer micro-benchmarks (profiling runs of the keystroke only)")
    ap.add_argument("--kernel-case",
                    choices=["linears", "mixer", "decode_step"] + [f"gemm_m{m}" for m in PREFILL_GEMM_ROWS]
                    + ["prefill_attn_t13", "prefill_attn_t32", "prefill_attn_t64", "prefill_attn_t256"],
                    help="run one small single-kernel workload for a full ncu capture, then exit")
    args = ap.parse_args()
    if args.kernel_case:
        kernel_case(args.kernel_case)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        if rank != 0:
            return
        try:
            cpu = run_reference(args.steps, args.warmup)
        except FileNotFoundError:  # no baseline/_ref install: the oracle port stands in
            cpu = run_port(args.steps, args.warmup)
        print(json.dumps({
            "impl": "reference",
            "metric": "Top-3 keystroke latency p50/p95 ms (8 cand), decode tok/s, mixer HBM GB/s",
            "value": round(cpu["value"], 4), "unit": "keystrokes/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 / cpu["value"], 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded random weights, seeded prefixes, synthetic tokenizer)",
            "config": bench_config(world),
            "latency_ms": {"p50": round(cpu["p50_ms"], 3), "p95": round(cpu["p95_ms"], 3)},
            "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(cpu["value"], 4), "unit": "keystrokes/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }))
        return
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        # replicas: the barrier and the max-over-ranks timing reduction are host-side
        # (gloo); no collective touches the GPUs
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=300))
        pin_rank_cores(local_rank, int(os.environ.get("LOCAL_WORLD_SIZE", world)))
    line = run_gpu(args, rank, world, local_rank)
    if rank == 0 and line is not None:
        if world == 1 and args.cpu_sample > 0:
            line["cpu_baseline"] = reference_subprocess(args.cpu_sample)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
