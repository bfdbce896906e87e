"""Asynchronous, layer-ordered store / load (cache_store_async,
cache_load_async, cache_async_*) on the CPU (MEM) backend: layer ranges land
at the right record offsets (oracle), a store publishes only complete
records, a load of a layer subset writes only those layers."""
import errno

import numpy as np
import pytest

from demo_b200 import cache as cc
from demo_b200._lib import CACHE_BACKEND_MEM
from oracle import kvcopy as ok
from tests.golden import gen
from tests.test_cache_host import HostKV, keys_for

CASE = dict(next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16"), num_layers=5)
BPC = CASE["chunk_size"] // CASE["block_size"]
REC = gen.record_bytes(CASE)
UNIT = gen.unit_of(CASE)


@pytest.fixture
def mem(tmp_path):
    def _init(records=8, disk=False):
        cc.init(CASE["chunk_size"], records * REC, str(tmp_path / "kv") if disk else None, CACHE_BACKEND_MEM)
        return tmp_path / "kv"
    yield _init
    cc.exit()


def expected(src, bids, dst_bids, layers=None):
    recs = ok.gather(src.k, src.v, bids, CASE["chunk_size"], CASE["block_size"], UNIT)
    k0, v0 = gen.paged_layers(CASE, zero=True)
    ok.scatter(recs, k0, v0, dst_bids, CASE["chunk_size"], CASE["block_size"], UNIT)
    if layers is not None:      # only these layers were loaded
        for l in range(CASE["num_layers"]):
            if l not in layers:
                k0[l][:] = 0
                v0[l][:] = 0
    return k0, v0


def same(dst, k0, v0):
    return all(np.array_equal(a, b) for a, b in zip(dst.k, k0)) and \
        all(np.array_equal(a, b) for a, b in zip(dst.v, v0))


def test_layered_store_then_sync_load(mem):
    mem()
    src = HostKV(CASE)
    w = src.worker()
    w.register()
    keys = keys_for(CASE["chunks"], seed=31)
    bids = gen.block_ids(CASE)
    h = w.store_async(keys, bids)
    assert h.records == CASE["chunks"] and not h.missing
    assert w.lookup(keys) == 0                     # reserved, not visible yet
    for l0, l1 in ((0, 2), (2, 3), (3, 5)):        # layer groups, in order
        h.layers(l0, l1)
    assert h.query()
    assert h.finish() == 0
    assert w.lookup(keys) == 32 * CASE["chunks"]
    st = w.stats()
    assert st["stored"] == CASE["chunks"] and st["bytes_saved"] == CASE["chunks"] * REC
    dst = HostKV(CASE, zero=True)
    wd = dst.worker()
    wd.register()
    b2 = gen.block_ids(CASE, seed_offset=1)
    assert wd.load(keys, b2) == 0
    assert same(dst, *expected(src, bids, b2))
    wd.unregister()
    w.unregister()


def test_store_missing_a_layer_is_dropped(mem):
    mem()
    src = HostKV(CASE)                 # the paged layers must outlive the worker
    w = src.worker()
    w.register()
    keys = keys_for(2, seed=32)
    h = w.store_async(keys, gen.block_ids(CASE)[:2 * BPC])
    h.layers(0, 2)
    h.layers(3, 5)                                  # layer 2 never copied
    assert h.finish() == -errno.EINVAL
    assert w.lookup(keys) == 0 and w.stats()["records_used"] == 0
    # a key already cached is skipped by a later async store
    assert w.store(keys[:1], gen.block_ids(CASE)[:BPC]) == 0
    h = w.store_async(keys, gen.block_ids(CASE)[:2 * BPC])
    assert h.records == 1 and w.stats()["store_dedup"] == 1
    h.layers(0, 5)
    assert h.finish() == 0
    assert w.lookup(keys) == 64
    w.unregister()


@pytest.mark.parametrize("ranges", [[(0, 5)], [(0, 1), (1, 2), (2, 3), (3, 4), (4, 5)], [(1, 3)], [(4, 5), (0, 1)]])
def test_layered_load_writes_exactly_those_layers(mem, ranges):
    mem()
    src, dst = HostKV(CASE), HostKV(CASE, zero=True)
    ws, wd = src.worker(), dst.worker()
    ws.register()
    wd.register()
    keys = keys_for(CASE["chunks"], seed=33)
    bids, b2 = gen.block_ids(CASE), gen.block_ids(CASE, seed_offset=1)
    assert ws.store(keys, bids) == 0
    h = wd.load_async(keys, b2)
    assert h.records == CASE["chunks"]
    for l0, l1 in ranges:
        h.layers(l0, l1)
    loaded = {l for l0, l1 in ranges for l in range(l0, l1)}
    for l in range(CASE["num_layers"]):
        if l in loaded:
            h.stream_wait(l)
        else:
            with pytest.raises(cc.CacheError) as e:
                h.stream_wait(l)
            assert e.value.ret == -errno.ENOENT
    assert h.finish() == 0
    assert same(dst, *expected(src, bids, b2, layers=loaded))
    assert wd.stats()["loaded"] == CASE["chunks"]
    wd.unregister()
    ws.unregister()


def test_load_async_skips_misses_and_checks_arguments(mem):
    mem()
    src, dst = HostKV(CASE), HostKV(CASE, zero=True)
    ws, wd = src.worker(), dst.worker()
    ws.register()
    wd.register()
    keys = keys_for(3, seed=34)
    bids = gen.block_ids(CASE)
    assert ws.store(keys[:1] + keys[2:], np.concatenate([bids[:BPC], bids[2 * BPC:3 * BPC]])) == 0
    h = wd.load_async(keys, bids)
    assert h.missing and h.records == 2
    with pytest.raises(cc.CacheError):
        h.layers(3, 3)                              # empty range
    with pytest.raises(cc.CacheError):
        h.layers(0, 6)                              # past the last layer
    with pytest.raises(cc.CacheError):
        h.layers(0, 5, stream=1)                    # the CPU backend takes no stream
    h.layers(0, 5)
    assert h.finish() == 0
    sel = np.concatenate([bids[:BPC], bids[2 * BPC:3 * BPC]])
    k0, v0 = expected(src, sel, sel)
    assert same(dst, k0, v0)
    # a block id past the paged cache fails the handle, pins are released
    h = wd.load_async(keys[:1], np.full(BPC, 10_000, np.uint64))
    h.layers(0, 5)
    assert h.finish() == -errno.EINVAL
    assert wd.stats()["records_used"] == 2
    wd.clear()
    assert wd.stats()["records_used"] == 0
    wd.unregister()
    ws.unregister()


def test_async_store_reaches_the_disk_tier(mem):
    root = mem(disk=True)
    src = HostKV(CASE)
    w = src.worker()
    w.register()
    keys = keys_for(2, seed=35)
    h = w.store_async(keys, gen.block_ids(CASE)[:2 * BPC])
    h.layers(0, 5)
    assert h.finish() == 0
    w.flush()
    assert w.stats()["disk_writes"] == 2
    recs = ok.gather(src.k, src.v, gen.block_ids(CASE)[:2 * BPC], CASE["chunk_size"], CASE["block_size"], UNIT)
    for k, r in zip(keys, recs):
        assert (root / "m.tp1.0" / k.hex()).read_bytes() == r.tobytes()
    w.unregister()
