"""CPU, world size 2 over gloo: the data-parallel logic of bench.py.

Sequences are sharded across ranks (each rank owns its own pool, seeded by
rank); the only collectives are the barrier and the max-over-ranks of the
timed region. Run as two spawned processes on 127.0.0.1.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "vllm-inference-engine_b200"))
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = bench.build_shard(rank, None, num_seqs=8, ctx=256, num_blocks=256)
        # per-rank pools / tables differ; within a rank every block appears once
        tables = shard["tables"]
        assert tables.unique().numel() == tables.numel()
        digest = int(tables.sum()) * 1000003 + int(shard["q"].float().sum().item() * 1000)
        dist.barrier()
        t = bench._max_over_ranks(dist, 1.5 + rank, torch.device("cpu"))
        s = bench._sum_over_ranks(dist, 10.0 * (rank + 1), torch.device("cpu"))
        out_q.put((rank, digest, t, s))
    finally:
        dist.destroy_process_group()


def test_dp_two_ranks_shard_and_reduce_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert res[0][1] != res[1][1], "ranks must own different shards"
    assert res[0][2] == res[1][2] == pytest.approx(2.5)  # max over ranks
    assert res[0][3] == res[1][3] == pytest.approx(30.0)
