"""Mixed-operation stress on the CUDA backend: threads share one (model, tp)
entry with a small pool and the disk tier on, and interleave synchronous,
layer-wise (async, on per-thread streams) and batched stores and loads.
Every load that reports success must reproduce the source blocks exactly."""
import errno
import threading

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from tests.golden import gen
from tests.gpu_util import DeviceKV
from tests.test_gpu_cache import keys_for, worker

pytestmark = pytest.mark.gpu

CASE = dict(next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16"), num_layers=3, num_blocks=128)
BPC = CASE["chunk_size"] // CASE["block_size"]
OK_FAIL = (0, -errno.ENOENT, -errno.ENOMEM)


def _rows(kv, bids):
    idx = torch.as_tensor(np.asarray(bids, np.int64), device="cuda")
    return [t.view(CASE["num_blocks"], -1)[idx] for t in kv.k + kv.v]


def test_mixed_operations_on_the_gpu(tmp_path):
    cc.init(CASE["chunk_size"], 6 * gen.record_bytes(CASE), str(tmp_path / "kv"))
    errors, stats = [], []
    try:
        def run(t):
            try:
                rng = np.random.default_rng(1900 + t)
                stream = torch.cuda.Stream()
                src = DeviceKV(CASE, seed=1300 + t)
                ws = worker(src)
                ws.register()
                keys = keys_for(8, seed=1700 + t)
                stored = set()
                for it in range(30):
                    c = int(rng.integers(0, 8))
                    b = np.arange(c * BPC, (c + 1) * BPC, dtype=np.uint64)
                    op = it % 3
                    if op == 0:
                        ret = ws.store([keys[c]], b)
                    elif op == 1:
                        h = ws.store_async([keys[c]], b)
                        for l in range(CASE["num_layers"]):
                            h.layers(l, l + 1, stream=stream)
                        ret = h.finish()
                    else:
                        ret, _ = ws.store_batch([[keys[c]]], [b])
                    assert ret in OK_FAIL, ("store", op, ret)
                    if ret == 0:
                        stored.add(c)
                    if not stored:
                        continue
                    j = int(rng.choice(sorted(stored)))
                    dst = DeviceKV(CASE, zero=True)
                    wd = worker(dst)
                    wd.register()
                    db = np.arange(((j + 1) % 8) * BPC, ((j + 1) % 8 + 1) * BPC, dtype=np.uint64)
                    how = it % 3
                    if how == 0:
                        ret = wd.load([keys[j]], db)
                    elif how == 1:
                        h = wd.load_async([keys[j]], db)
                        if h.records:
                            for l in range(CASE["num_layers"]):
                                h.layers(l, l + 1, stream=stream)
                        ret = h.finish() if h.records else -errno.ENOENT
                    else:
                        ret, _ = wd.load_batch([[keys[j]]], [db])
                    assert ret in OK_FAIL, ("load", how, ret)
                    if ret == 0:
                        torch.cuda.synchronize()
                        sb = np.arange(j * BPC, (j + 1) * BPC)
                        for a, e in zip(_rows(dst, db), _rows(src, sb)):
                            assert torch.equal(a, e), (t, it, j, how)
                    wd.unregister()
                ws.flush()
                stats.append(ws.stats())
                ws.unregister()
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append((t, repr(e)))

        ths = [threading.Thread(target=run, args=(t,)) for t in range(4)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
    finally:
        cc.exit()
    assert not errors, errors
    last = max(stats, key=lambda s: s["stored"])
    assert last["evictions"] > 0 and last["disk_reads"] > 0
