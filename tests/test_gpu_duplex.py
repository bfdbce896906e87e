"""The pipelined duplex pattern the bench's value step runs, through the cache
API on the CUDA backend: step k stores batch k on one thread while two
threads load batch k-1 (saved one step earlier), with a pool of three
batches, so saves (D2H) and loads (H2D) share the host link and LRU eviction
runs from the third step on.  Every step checks the reloaded blocks byte for
byte, every load must hit (LRU must never evict the batch about to be
loaded), and the eviction count must be what the pool size gives."""
import threading

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from tests.golden import gen
from tests.gpu_util import DeviceKV

pytestmark = pytest.mark.gpu

CASE = dict(name="duplex", num_blocks=256, block_size=16, chunk_size=256, num_layers=4, hidden=1024, elt=2,
            kv=2, chunks=8, seed=21)
REQS, KPR = 4, 2                                  # requests per batch, records per request
PRB = KPR * CASE["chunk_size"] // CASE["block_size"]


def _keys(step: int) -> list[bytes]:
    rng = np.random.default_rng(1000 + step)
    return [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(REQS * KPR)]


def _blocks(t: torch.Tensor) -> torch.Tensor:
    return t.view(CASE["num_blocks"], -1)


def test_store_batch_k_while_two_threads_load_batch_k_minus_1():
    kv = DeviceKV(CASE)
    rec = gen.record_bytes(CASE)
    perm = np.random.default_rng(5).permutation(CASE["num_blocks"]).astype(np.uint64)
    save, load = perm[:REQS * PRB], perm[REQS * PRB:2 * REQS * PRB]
    idx_s = torch.from_numpy(save.astype(np.int64)).cuda()
    idx_l = torch.from_numpy(load.astype(np.int64)).cuda()
    planes = kv.k + kv.v
    for t in planes:
        _blocks(t)[idx_l] = 0
    torch.cuda.synchronize()
    cc.init(CASE["chunk_size"], (3 * REQS * KPR + 1) * rec, None)
    try:
        lay = cc.KVLayout(CASE["num_layers"], CASE["num_blocks"], CASE["block_size"], CASE["hidden"],
                          CASE["elt"], CASE["kv"])
        w = cc.Worker("duplex", lay, [t.data_ptr() for t in kv.k], [t.data_ptr() for t in kv.v],
                      node_id=torch.cuda.current_device())
        w.register()
        total = w.stats()["records_total"]
        assert w.store(_keys(0), save) == 0                      # batch 0, before the first step
        for k in range(1, 7):
            kb, prev = _keys(k), _keys(k - 1)
            assert w.lookup(prev) == 32 * REQS * KPR             # the whole previous batch is there
            rets: list = []

            def saver():
                for r in range(REQS):
                    rets.append(w.store(kb[r * KPR:(r + 1) * KPR], save[r * PRB:(r + 1) * PRB]))

            def loader(j):
                for r in range(j, REQS, 2):
                    rets.append(w.load(prev[r * KPR:(r + 1) * KPR], load[r * PRB:(r + 1) * PRB]))

            ths = [threading.Thread(target=saver)] + [threading.Thread(target=loader, args=(j,)) for j in range(2)]
            for t in ths:
                t.start()
            for t in ths:
                t.join()
            assert rets == [0] * (2 * REQS), (k, rets)
            torch.cuda.synchronize()
            for t in planes:                                     # batch k-1 = the save blocks' bytes
                assert torch.equal(_blocks(t)[idx_s], _blocks(t)[idx_l]), k
            st = w.stats()
            assert st["evictions"] == max(0, (k + 1) * REQS * KPR - total), (k, st)
            assert st["loaded"] == k * REQS * KPR, (k, st)
        w.unregister()
    finally:
        cc.exit()
