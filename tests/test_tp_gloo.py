"""TP agreement on CPU: two gloo ranks, each with its own head-shard pool
(MEM backend), agree the per-request hit length with all-reduce(min) and
load exactly that many records (no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    from demo_b200 import cache as cc
    from demo_b200._lib import CACHE_BACKEND_MEM
    from demo_b200.tp import agree_min_hits, head_shard
    from tests.golden import gen

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        h0, h1 = head_shard(8, world, rank)
        case = dict(num_blocks=64, block_size=16, chunk_size=256, num_layers=2, hidden=(h1 - h0) * 128,
                    elt=2, kv=2, chunks=1, seed=40 + rank)
        cc.init(256, 16 * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
        k, v = gen.paged_layers(case)
        lay = cc.KVLayout(2, 64, 16, case["hidden"], 2, 2)
        w = cc.Worker("tp-model", lay, [a.ctypes.data for a in k], [a.ctypes.data for a in v],
                      world_size=world, rank=rank)
        w.register()
        rng = np.random.default_rng(0)                       # same keys on every rank
        reqs = [[rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(3)] for _ in range(4)]
        # rank r cached a different prefix length of each request
        cached = [[3, 1, 0, 2], [2, 3, 0, 1]][rank]
        for keys, n in zip(reqs, cached):
            if n:
                assert w.store(keys[:n], np.arange(16 * n, dtype=np.uint64)) == 0
        local = w.lookup_batch(reqs)
        agreed = agree_min_hits(local)
        # every rank loads the agreed number of records
        for keys, n in zip(reqs, agreed):
            assert w.load(keys[: int(n)], np.arange(16 * int(n), 32 * int(n), dtype=np.uint64)) == 0
        q.put((rank, local.tolist(), agreed.tolist(), w.stats()["loaded"]))
        w.unregister()
        cc.exit()
    finally:
        dist.destroy_process_group()


def test_two_rank_min_hit_agreement():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert res[0][1] == [3, 1, 0, 2] and res[1][1] == [2, 3, 0, 1]
    assert res[0][2] == res[1][2] == [2, 1, 0, 1]
    assert res[0][3] == res[1][3] == 4


def test_head_shard_split():
    from demo_b200.tp import head_shard

    assert [head_shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        head_shard(8, 3, 0)
