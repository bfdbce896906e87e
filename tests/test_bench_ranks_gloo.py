"""bench.py's multi-rank aggregation on CPU: two gloo ranks take the Ranks
collectives (barrier, max, min, sum, gather) that produce every N > 1 number
of the bench line -- the slowest rank's time, the agreed request count, the
summed payload, the per-GPU link rates -- in the same order on every rank."""
import os
import socket

import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, world: int, port: int, q):
    import sys

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.environ["BENCH_ROOT"])
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rk = bench.Ranks(world, rank, rank, torch.device("cpu"), world, rank)
        rk.barrier()
        x = 10.0 * (rank + 1)                       # 10 on rank 0, 20 on rank 1
        out = (rk.max(x), rk.min(x), rk.sum(x), rk.gather(x))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_ranks_collectives_on_two_gloo_ranks():
    from pathlib import Path
    os.environ["BENCH_ROOT"] = str(Path(__file__).resolve().parent.parent)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        mx, mn, sm, g = res[r]
        assert (mx, mn, sm) == (20.0, 10.0, 30.0)
        assert g == [10.0, 20.0]


def test_ranks_single_process_is_the_identity():
    import sys
    from pathlib import Path

    import torch
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import bench
    rk = bench.Ranks(1, 0, 0, torch.device("cpu"), 1, 0)
    rk.barrier()
    assert (rk.max(3.5), rk.min(3.5), rk.sum(3.5), rk.gather(3.5)) == (3.5, 3.5, 3.5, [3.5])
