"""CPU: the data-parallel request router (least outstanding tokens, prefix
affinity) and its trace form, including two gloo ranks computing the same
assignment without exchanging anything but the check."""
import os
import socket
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from pagedkv.router import RequestRouter, route_trace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_equal_requests_spread_round_robin():
    r = RequestRouter(4)
    assert [r.assign(100) for _ in range(8)] == [0, 1, 2, 3, 0, 1, 2, 3]
    assert r.load == [200, 200, 200, 200]


def test_least_outstanding_tokens_wins_and_release_counts():
    r = RequestRouter(3)
    assert r.assign(1000) == 0
    assert r.assign(10) == 1
    assert r.assign(10) == 2
    assert r.assign(10) == 1  # ranks 1 and 2 tie at 10: the lower rank wins
    r.release(0, 1000)
    assert r.assign(5) == 0
    with pytest.raises(ValueError):
        r.release(2, 11)
    with pytest.raises(ValueError):
        r.release(3, 1)


def test_prefix_affinity_until_the_slack_is_exceeded():
    r = RequestRouter(2, affinity_slack=250)
    assert r.assign(100, "g") == 0
    assert r.assign(100, "g") == 0  # home rank 0 is 100 above rank 1: within the slack
    assert r.assign(100, "g") == 0  # 200 above
    assert r.assign(100, "g") == 1  # 300 above: spills to the least loaded rank
    assert r.assign(100, "h") == 1 and r.prefix_rank["h"] == 1
    assert r.prefix_rank["g"] == 0


def test_config4_groups_stay_on_one_rank_each():
    # 8 groups x 64 sequences of 1280 tokens, arriving group-interleaved
    keys = [g for _ in range(64) for g in range(8)]
    ranks = route_trace([1280] * len(keys), 8, keys)
    home = {}
    for k, rk in zip(keys, ranks):
        assert home.setdefault(k, rk) == rk
    assert sorted(home.values()) == list(range(8))


def test_route_trace_is_deterministic_and_balanced():
    import random

    rnd = random.Random(3)
    tokens = [rnd.randint(64, 1024) + 128 for _ in range(2000)]
    a = route_trace(tokens, 8)
    assert a == route_trace(tokens, 8)
    loads = [0] * 8
    for t, rk in zip(tokens, a):
        loads[rk] += t
    assert max(loads) - min(loads) <= max(tokens)
    with pytest.raises(ValueError):
        route_trace(tokens, 8, prefix_keys=[None])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_q):
    sys.path.insert(0, os.path.join(ROOT, "vllm-inference-engine_b200"))
    import random

    from pagedkv.router import route_trace as rt

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rnd = random.Random(11)  # the same global trace on every rank
        tokens = [rnd.randint(64, 1024) + 128 for _ in range(500)]
        mine = [i for i, rk in enumerate(rt(tokens, world)) if rk == rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        out_q.put((rank, gathered, len(tokens)))
    finally:
        dist.destroy_process_group()


def test_two_ranks_take_disjoint_shares_of_one_trace():
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
    (_, g0, n), (_, g1, _) = res
    assert g0 == g1
    shares = g0
    assert sorted(shares[0] + shares[1]) == list(range(n))
    assert not set(shares[0]) & set(shares[1])
