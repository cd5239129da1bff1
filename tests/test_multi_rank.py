"""Multi-process host logic of the request partition, on CPU ranks (gloo, world size 2).

The GPU path shards independent sequences over ranks with no data-path collective; only
the timing gather crosses ranks.  These tests run that plumbing as two gloo processes:
every sequence is owned by exactly one rank, the max/sum gathers bench.py uses agree on all
ranks, and a rank that dies before a collective makes the survivor fail fast instead of
hanging (failure injected on the host: a worker that raises).
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _paths():
    for sub in ("dory-vllm-experiments_b200", ""):
        p = str(ROOT / sub) if sub else str(ROOT)
        if p not in sys.path:
            sys.path.insert(0, p)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _partition_worker(rank, world, port, queue):
    _paths()
    import bench
    import workloads as W
    dist = _init(rank, world, port, 60)
    lens = W.config5_lens()
    mine = W.partition(lens, world)[rank]
    owned = torch.zeros(len(lens), dtype=torch.int64)
    owned[mine] = 1
    dist.all_reduce(owned)
    tokens = float(sum(lens[i] + 1 for i in mine))
    cpu = torch.device("cpu")
    mx = bench.max_over_ranks(dist, tokens, cpu)
    total = bench.sum_over_ranks(dist, tokens, cpu)
    queue.put((rank, owned.tolist(), tokens, mx, total))
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, queue):
    _paths()
    import bench
    dist = _init(rank, world, port, 10)
    if rank == 1:
        os._exit(3)  # dies between steps, before the timing gather
    try:
        bench.max_over_ranks(dist, 1.0, torch.device("cpu"))
        queue.put((rank, "completed"))
    except Exception as e:  # gloo reports the lost peer
        queue.put((rank, f"detected: {type(e).__name__}"))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not queue.empty():
        out.append(queue.get())
    return out, procs, alive


def test_request_partition_over_two_ranks():
    _paths()
    import workloads as W
    out, procs, alive = _run(_partition_worker)
    assert not alive
    assert all(p.exitcode == 0 for p in procs)
    assert len(out) == 2
    lens = W.config5_lens()
    for rank, owned, tokens, mx, total in out:
        assert owned == [1] * len(lens)  # every sequence on exactly one rank
        assert total == sum(n + 1 for n in lens)
        assert mx == max(o[2] for o in out)
    # token-balanced: the two shares differ by at most one longest request
    shares = sorted(o[2] for o in out)
    assert shares[1] - shares[0] <= max(lens) + 1


def test_dead_rank_is_detected_not_hung():
    out, procs, alive = _run(_failing_worker, timeout=90)
    assert not alive, "the surviving rank hung"
    survivor = [o for o in out if o[0] == 0]
    assert survivor and survivor[0][1].startswith("detected"), out
