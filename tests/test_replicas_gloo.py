"""The multi-GPU bench path on the CPU: `bench.py --gpus N` runs N independent
keystroke replicas, and the only cross-rank steps are a barrier and the
max-over-ranks reduction of the timed region, both host-side over gloo. Two gloo
ranks (separate processes, 127.0.0.1) check that reduction, the per-rank
gather and the whole-job throughput, and the core pinning of each rank."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]

_RANK_CODE = r"""
import json, os, sys
from datetime import timedelta
sys.path.insert(0, os.environ["REPO"])
import torch
import torch.distributed as dist
import bench
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
try:
    # rank r timed device_ms = 100 + 40 r and wall = 0.5 - 0.1 r
    got = bench.max_over_ranks([100.0 + 40.0 * rank, 0.5 - 0.1 * rank], world)
    per_rank = bench.gather_over_ranks(3.0 + rank, world)
    dist.barrier()
    print(json.dumps({"rank": rank, "max": got, "per_rank": per_rank,
                      "value": bench.replica_throughput(world, 30, got[0])}))
finally:
    dist.destroy_process_group()
"""


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_replicas_reduce_timings_to_the_slowest_rank() -> None:
    world = 2
    env = dict(os.environ, REPO=str(REPO), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()),
               WORLD_SIZE=str(world), CUDA_VISIBLE_DEVICES="")
    procs = [subprocess.Popen([sys.executable, "-c", _RANK_CODE], env=dict(env, RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=120)
        finally:
            if p.poll() is None:
                p.kill()
        assert p.returncode == 0, err[-2000:]
        outs.append(json.loads(out.strip().splitlines()[-1]))
    assert sorted(o["rank"] for o in outs) == [0, 1]
    for o in outs:
        # every rank sees the slowest replica's time, and value counts all replicas
        assert o["max"] == [140.0, 0.5]
        assert o["per_rank"] == [3.0, 4.0]
        assert abs(o["value"] - world * 30 / 0.140) < 1e-9


def test_rank_core_pinning_splits_the_host_cores() -> None:
    code = ("import os, sys, json; sys.path.insert(0, os.environ['REPO']); import bench; "
            "print(json.dumps([bench.pin_rank_cores(r, 2) for r in (0,)] + [sorted(os.sched_getaffinity(0))]))")
    out = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, REPO=str(REPO)), capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    mine, now = json.loads(out.stdout.strip().splitlines()[-1])
    allowed = sorted(os.sched_getaffinity(0))
    assert now == mine and set(mine) <= set(allowed)
    assert len(mine) == max(1, len(allowed) // 2)


def test_single_rank_reduction_is_the_identity() -> None:
    sys.path.insert(0, str(REPO))
    import torch

    import bench

    assert bench.max_over_ranks([3.25, 1.5], 1, torch.device("cpu")) == [3.25, 1.5]
    assert bench.replica_throughput(1, 30, 100.0) == 300.0
