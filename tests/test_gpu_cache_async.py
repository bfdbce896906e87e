"""Asynchronous layer-ordered store / load on the GPU: copies enqueued per
layer on a side stream, a compute stream that waits (on the GPU) for each
layer before reading it, a store gated on an event recorded after the
compute stream rewrote the layer.  Bytes against the oracle."""
import errno

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from demo_b200._lib import lib
from oracle import kvcopy as ok
from tests.golden import gen
from tests.gpu_util import DeviceKV
from tests.test_gpu_cache import keys_for, worker

pytestmark = pytest.mark.gpu

CASE = dict(next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16"), num_layers=6, num_blocks=256, chunks=8)
BPC = CASE["chunk_size"] // CASE["block_size"]
UNIT = gen.unit_of(CASE)


@pytest.fixture
def cuda_cache():
    cc.init(CASE["chunk_size"], (2 * CASE["chunks"] + 2) * gen.record_bytes(CASE), None)
    yield
    cc.exit()


def _expected(bids, dst_bids):
    k, v = gen.paged_layers(CASE)
    recs = ok.gather(k, v, bids, CASE["chunk_size"], CASE["block_size"], UNIT)
    ek, ev = gen.paged_layers(CASE, zero=True)
    ok.scatter(recs, ek, ev, dst_bids, CASE["chunk_size"], CASE["block_size"], UNIT)
    return ek, ev


def test_layerwise_load_with_gpu_side_waits(cuda_cache):
    src, dst = DeviceKV(CASE), DeviceKV(CASE, zero=True)
    ws, wd = worker(src), worker(dst)
    ws.register()
    wd.register()
    keys = keys_for(CASE["chunks"], seed=41)
    bids, b2 = gen.block_ids(CASE), gen.block_ids(CASE, seed_offset=1)
    assert ws.store(keys, bids) == 0
    ek, ev = _expected(bids, b2)
    load_stream, compute = torch.cuda.Stream(), torch.cuda.Stream()
    n0 = lib.crosscache_kernel_launches()
    h = wd.load_async(keys, b2)
    assert h.records == CASE["chunks"] and not h.missing
    for l in range(CASE["num_layers"]):
        h.layers(l, l + 1, stream=load_stream)
    # the compute stream reads each layer right after its GPU-side wait
    sums = []
    with torch.cuda.stream(compute):
        for l in range(CASE["num_layers"]):
            h.stream_wait(l, compute)
            sums.append((dst.k[l].to(torch.int64).sum(), dst.v[l].to(torch.int64).sum()))
    compute.synchronize()
    assert h.finish() == 0
    assert lib.crosscache_kernel_launches() - n0 == CASE["num_layers"]
    for l in range(CASE["num_layers"]):
        assert int(sums[l][0]) == int(ek[l].astype(np.int64).sum()), l
        assert int(sums[l][1]) == int(ev[l].astype(np.int64).sum()), l
    kh, vh = dst.host()
    assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
    assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
    wd.unregister()
    ws.unregister()


def test_layerwise_store_gated_on_compute_events(cuda_cache):
    """the compute stream rewrites each layer, records an event, and the
    store of that layer waits for it: the records hold the new bytes"""
    src = DeviceKV(CASE, zero=True)
    ws = worker(src)
    ws.register()
    keys = keys_for(CASE["chunks"], seed=42)
    bids = gen.block_ids(CASE)
    k_new, v_new = gen.paged_layers(CASE, seed=777)
    save_stream, compute = torch.cuda.Stream(), torch.cuda.Stream()
    h = ws.store_async(keys, bids)
    assert h.records == CASE["chunks"]
    host_k = [torch.from_numpy(a).pin_memory() for a in k_new]
    host_v = [torch.from_numpy(a).pin_memory() for a in v_new]
    for l in range(CASE["num_layers"]):
        with torch.cuda.stream(compute):
            torch.cuda._sleep(2_000_000)          # the "layer" takes a while
            src.k[l].copy_(host_k[l], non_blocking=True)
            src.v[l].copy_(host_v[l], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(compute)
        h.layers(l, l + 1, stream=save_stream, wait_event=ev)
    assert ws.lookup(keys) == 0
    assert h.finish() == 0
    assert ws.lookup(keys) == 32 * CASE["chunks"]
    # load the records into a zeroed cache and compare with the new bytes
    dst = DeviceKV(CASE, zero=True)
    wd = worker(dst)
    wd.register()
    b2 = gen.block_ids(CASE, seed_offset=1)
    assert wd.load(keys, b2) == 0
    recs = ok.gather(k_new, v_new, bids, CASE["chunk_size"], CASE["block_size"], UNIT)
    ek, ev_ = gen.paged_layers(CASE, zero=True)
    ok.scatter(recs, ek, ev_, b2, CASE["chunk_size"], CASE["block_size"], UNIT)
    kh, vh = dst.host()
    assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
    assert all(np.array_equal(a, b) for a, b in zip(vh, ev_))
    wd.unregister()
    ws.unregister()


def test_async_errors(cuda_cache):
    src = DeviceKV(CASE)
    ws = worker(src)
    ws.register()
    keys = keys_for(2, seed=43)
    bids = gen.block_ids(CASE)[:2 * BPC]
    assert ws.store(keys, bids) == 0
    s = torch.cuda.Stream()
    # a block id past the paged cache: the kernel flags it, finish reports it
    h = ws.load_async(keys[:1], np.full(BPC, 1 << 40, np.uint64))
    h.layers(0, CASE["num_layers"], stream=s)
    assert h.finish() == -errno.EINVAL
    # a store that never enqueued its last layer is dropped
    fresh = keys_for(1, seed=44)
    h = ws.store_async(fresh, bids[:BPC])
    h.layers(0, CASE["num_layers"] - 1, stream=s)
    assert h.finish() == -errno.EINVAL
    assert ws.lookup(fresh) == 0
    # nothing pinned or pending is left behind
    st = ws.stats()
    assert st["records_used"] == 2
    ws.clear()
    assert ws.stats()["records_used"] == 0
    ws.unregister()


def test_layerwise_copies_on_a_fragmented_pool():
    """records of one handle in descending runs (slabs freed by a clear come
    back last-first), ascending runs and singletons: the copy engine moves
    runs with one command each; every byte lands where the oracle says"""
    case = dict(CASE, num_blocks=512, chunks=12)
    rec = gen.record_bytes(case)
    cc.init(case["chunk_size"], 12 * rec, None)
    try:
        src = DeviceKV(case)
        ws = worker(src)
        ws.register()
        bids = gen.block_ids(case)
        a_keys, b_keys, c_keys = keys_for(8, seed=61), keys_for(8, seed=62), keys_for(3, seed=63)
        assert ws.store(a_keys, bids[:8 * BPC]) == 0          # slabs 0..7
        ws.clear()
        s = torch.cuda.Stream()
        # async store into slabs 7, 6, ..., 0 (descending)
        h = ws.store_async(b_keys, bids[:8 * BPC])
        h.layers(0, CASE["num_layers"], stream=s)
        assert h.finish() == 0
        assert ws.store(c_keys, bids[8 * BPC:11 * BPC]) == 0   # slabs 8, 9, 10
        pick = [(b_keys, 0), (c_keys, 0), (b_keys, 1), (c_keys, 1), (b_keys, 5), (b_keys, 2), (c_keys, 2),
                (b_keys, 7)]
        keys = [k[i] for k, i in pick]
        src_chunks = [i if k is b_keys else 8 + i for k, i in pick]
        dst = DeviceKV(case, zero=True)
        wd = worker(dst)
        wd.register()
        b2 = gen.block_ids(case, seed_offset=1)[:len(pick) * BPC]
        h = wd.load_async(keys, b2)
        assert h.records == len(pick)
        for l in range(CASE["num_layers"]):
            h.layers(l, l + 1, stream=s)
        assert h.finish() == 0
        torch.cuda.synchronize()
        sel = np.concatenate([bids[c * BPC:(c + 1) * BPC] for c in src_chunks])
        k, v = gen.paged_layers(case)
        recs = ok.gather(k, v, sel, case["chunk_size"], case["block_size"], UNIT)
        ek, ev = gen.paged_layers(case, zero=True)
        ok.scatter(recs, ek, ev, b2, case["chunk_size"], case["block_size"], UNIT)
        kh, vh = dst.host()
        assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
        assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()


@pytest.mark.parametrize("name", ["mla_bs64", "tp8_shard", "test_copy_defaults"])
def test_layerwise_roundtrip_other_layouts(name):
    """K-only MLA latent (block 64, 1152-byte unit), a one-head TP shard
    (256-byte unit) and the reference test's defaults (block 2, 4-token
    records): layer-by-layer store into the pool, then layer-by-layer load
    into a zeroed cache at a second block table, bytes against the oracle"""
    case = next(c for c in gen.KV_CASES if c["name"] == name)
    unit = gen.unit_of(case)
    bpc = case["chunk_size"] // case["block_size"]
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), None)
    try:
        src, dst = DeviceKV(case), DeviceKV(case, zero=True)
        ws, wd = worker(src), worker(dst)
        ws.register()
        wd.register()
        keys = keys_for(case["chunks"], seed=71)
        bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
        s = torch.cuda.Stream()
        h = ws.store_async(keys, bids)
        for l in range(case["num_layers"]):
            h.layers(l, l + 1, stream=s)
        assert h.finish() == 0
        h = wd.load_async(keys, b2)
        assert h.records == case["chunks"]
        for l in reversed(range(case["num_layers"])):        # any layer order
            h.layers(l, l + 1, stream=s)
        assert h.finish() == 0
        torch.cuda.synchronize()
        k, v = gen.paged_layers(case)
        recs = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], unit)
        ek, ev = gen.paged_layers(case, zero=True)
        ok.scatter(recs, ek, ev, b2, case["chunk_size"], case["block_size"], unit)
        kh, vh = dst.host()
        assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
        if vh is not None:
            assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
        assert len(bids) == case["chunks"] * bpc
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()


def test_teardown_with_an_unfinished_handle_is_safe():
    """a handle enqueued and never finished: cache_exit lets its copies run
    out before unmapping anything (the entry keeps its pool), and the
    context stays usable for a new cache"""
    case = CASE
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), None)
    src = DeviceKV(case)
    ws = worker(src)
    ws.register()
    keys = keys_for(case["chunks"], seed=81)
    bids = gen.block_ids(case)
    assert ws.store(keys, bids) == 0
    dst = DeviceKV(case, zero=True)
    wd = worker(dst)
    wd.register()
    s = torch.cuda.Stream()
    h = wd.load_async(keys, gen.block_ids(case, seed_offset=1))
    for l in range(case["num_layers"]):
        h.layers(l, l + 1, stream=s)
    abandoned = h                      # never finished (finishing after exit is not allowed)
    wd.unregister()
    ws.unregister()
    cc.exit()
    torch.cuda.synchronize()
    # a fresh cache on the same device works
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), None)
    try:
        w2 = worker(src, name="m2")
        w2.register()
        assert w2.store(keys, bids) == 0
        assert w2.lookup(keys) == 32 * case["chunks"]
        w2.unregister()
    finally:
        cc.exit()
    del abandoned
