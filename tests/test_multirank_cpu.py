"""CPU, world size 2 over gloo: bench.py's replica aggregation (value = ranks * steps / slowest rank's
time; every rank decodes the same seeded workload)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        from cudallm_b200 import synth
        per_rank_ms = [100.0, 250.0][rank]
        q.put((rank, bench.max_over_ranks(per_rank_ms), bench.aggregate_tok_s(per_rank_ms, 256),
               synth.prompt_ids(32, seed=0), bench.dist_info()))
    finally:
        dist.destroy_process_group()


def test_replica_aggregation_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, tok_s, prompt, info in out:
        assert mx == 250.0
        assert tok_s == pytest.approx(2 * 256 / 0.25)
        assert prompt == out[0][3]
        assert info == (rank, 2, rank)
