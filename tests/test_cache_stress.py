"""Mixed-operation stress on the CPU (MEM) backend: threads share one
(model, tp) entry whose pool holds far fewer records than they store, with
the disk tier on, and interleave cache_store / cache_store_async /
cache_store_batch with cache_load / cache_load_async / cache_load_batch and
lookups.  Every load that reports success must produce exactly the source
bytes of its keys (eviction, write-behind pins, PENDING records and file
fallback all race here); failures may only be -ENOENT / -ENOMEM."""
import errno
import threading

import numpy as np

from demo_b200 import cache as cc
from demo_b200._lib import CACHE_BACKEND_MEM
from tests.golden import gen
from tests.test_cache_host import HostKV, keys_for

CASE = dict(next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16"), num_layers=2, num_blocks=128)
BPC = CASE["chunk_size"] // CASE["block_size"]
OK_FAIL = (0, -errno.ENOENT, -errno.ENOMEM)


def _blocks(kv, bids):
    return [a.reshape(CASE["num_blocks"], -1)[np.asarray(bids, np.int64)] for a in kv.k + kv.v]


def test_mixed_operations_keep_every_loaded_byte_right(tmp_path):
    cc.init(CASE["chunk_size"], 6 * gen.record_bytes(CASE), str(tmp_path / "kv"), CACHE_BACKEND_MEM)
    errors, stats = [], []
    try:
        def run(t):
            try:
                rng = np.random.default_rng(900 + t)
                src = HostKV(CASE, seed=300 + t)       # each thread its own source data ...
                ws = src.worker()
                ws.register()                          # ... all in the one shared entry
                keys = keys_for(8, seed=700 + t)       # and its own keys
                stored = set()
                for it in range(40):
                    c = int(rng.integers(0, 8))
                    b = np.arange(c * BPC, (c + 1) * BPC, dtype=np.uint64)
                    op = it % 3
                    if op == 0:
                        ret = ws.store([keys[c]], b)
                    elif op == 1:
                        h = ws.store_async([keys[c]], b)
                        h.layers(0, CASE["num_layers"])
                        ret = h.finish()
                    else:
                        ret, st = ws.store_batch([[keys[c]]], [b])
                    assert ret in OK_FAIL, ("store", op, ret)
                    if ret == 0:
                        stored.add(c)
                    if not stored:
                        continue
                    # load a stored chunk into a zeroed cache, verify the blocks
                    j = int(rng.choice(sorted(stored)))
                    dst = HostKV(CASE, zero=True)
                    wd = dst.worker()
                    wd.register()
                    db = np.arange(((j + 1) % 8) * BPC, ((j + 1) % 8 + 1) * BPC, dtype=np.uint64)
                    how = it % 3
                    if how == 0:
                        ret = wd.load([keys[j]], db)
                    elif how == 1:
                        h = wd.load_async([keys[j]], db)
                        if h.records:
                            h.layers(0, CASE["num_layers"])
                        ret = h.finish() if h.records else -errno.ENOENT
                    else:
                        ret, _ = wd.load_batch([[keys[j]]], [db])
                    assert ret in OK_FAIL, ("load", ret)
                    if ret == 0:
                        sb = np.arange(j * BPC, (j + 1) * BPC)
                        for a, e in zip(_blocks(dst, db), _blocks(src, sb)):
                            assert np.array_equal(a, e), (t, it, j)
                    wd.lookup(keys)
                    wd.unregister()
                ws.flush()
                stats.append(ws.stats())
                ws.unregister()
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append((t, repr(e)))

        ths = [threading.Thread(target=run, args=(t,)) for t in range(6)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
    finally:
        cc.exit()
    assert not errors, errors
    last = max(stats, key=lambda s: s["stored"])       # entry-wide counters
    print(last)
    # the run went through eviction, write-behind and the file fallback
    assert last["evictions"] > 0 and last["disk_writes"] > 0 and last["disk_reads"] > 0


def test_lookups_racing_with_the_last_unregister():
    """a lookup needs no registration of its own (the server answers them for
    rank 0 of a model): lookups in one thread while another registers and
    unregisters the entry's only worker must see either the entry or none,
    never a freed one"""
    import ctypes as C

    from demo_b200._lib import CacheStats, ModelInfo, WorkerContext, lib

    cc.init(CASE["chunk_size"], 2 * gen.record_bytes(CASE), None, CACHE_BACKEND_MEM)
    stop = threading.Event()
    errors = []
    try:
        keys = keys_for(4, seed=5)
        kb = b"".join(keys)
        name = b"m"

        def lookups():
            try:
                ctx = WorkerContext()
                ctx.model = ModelInfo(name, 0, 0, 0)
                ctx.world_size = 1
                ctx.rank_id = 0
                st = CacheStats()
                n = 0
                while not stop.is_set() or n < 1000:
                    r = lib.cache_lookup(C.byref(ctx), kb, 4, 32)
                    if r not in (0, 32, 64, 96, 128):
                        errors.append(r)
                    if lib.cache_get_stats(C.byref(ctx), C.byref(st)) not in (0, -errno.ENOENT):
                        errors.append("stats")
                    n += 1
                lookups.count = n
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append(repr(e))

        th = threading.Thread(target=lookups)
        th.start()
        src = HostKV(CASE)
        for i in range(200):
            w = src.worker()
            w.register()
            if i % 2:
                assert w.store(keys[:1], np.arange(BPC, dtype=np.uint64)) == 0
            w.unregister()
        stop.set()
        th.join()
    finally:
        stop.set()
        cc.exit()
    assert not errors, errors[:5]
    assert lookups.count >= 1000
