"""Disk tier of the cache manager through the public C API on the CPU (MEM)
backend: record files, their bytes against the reference digests and the
oracle, lookups and loads that fall back to files, persistence across
cache_exit / cache_init, missing and damaged files, per-rank namespaces."""
import errno
import hashlib
import os

import numpy as np
import pytest

from demo_b200 import cache as cc
from demo_b200._lib import CACHE_BACKEND_MEM
from oracle import kvcopy as ok
from tests.golden import gen
from tests.test_cache_host import HostKV, keys_for

CASE = next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16")     # 3 chunks, 4K-aligned records
BPC = CASE["chunk_size"] // CASE["block_size"]
REC = gen.record_bytes(CASE)


@pytest.fixture
def disk_cache(tmp_path):
    root = tmp_path / "kvfiles"

    def _init(records, chunk=None):
        cc.init(chunk or CASE["chunk_size"], records * REC, str(root), CACHE_BACKEND_MEM)
        return root
    yield _init
    cc.exit()


def ns_dir(root, model="m", world=1, rank=0):
    return root / f"{model}.tp{world}.{rank}"


def expected_scatter(src, keys_bids, dst_bids):
    """paged layers after loading the records of src's block ranges into a
    zeroed cache at dst_bids (oracle gather + scatter)"""
    case = src.case
    recs = ok.gather(src.k, src.v, keys_bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    k0, v0 = gen.paged_layers(case, zero=True)
    ok.scatter(recs, k0, v0, dst_bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    return k0, v0


def test_record_files_equal_reference_records(disk_cache, golden_records):
    """each stored record lands in <root>/<model>.tp1.0/<hex key> with the
    bytes CrossCache's own mem.cpp gathers (golden digests)"""
    root = disk_cache(CASE["chunks"] + 1)
    src = HostKV(CASE)
    w = src.worker()
    w.register()
    bids = gen.block_ids(CASE)
    keys = keys_for(CASE["chunks"], seed=1)
    assert w.store(keys, bids) == 0
    w.flush()
    st = w.stats()
    assert st["disk_writes"] == CASE["chunks"] and st["bytes_written_disk"] == CASE["chunks"] * REC
    files = sorted(p.name for p in ns_dir(root).iterdir())
    assert files == sorted(k.hex() for k in keys)                    # no temporaries left
    g = golden_records[CASE["name"]]
    for k, digest in zip(keys, g["record_sha256"]):
        data = (ns_dir(root) / k.hex()).read_bytes()
        assert len(data) == REC
        assert hashlib.sha256(data).hexdigest() == digest
    w.unregister()


def test_evicted_records_come_back_from_disk(disk_cache):
    """pool of 3 records, 6 stored in three calls: the first ones are evicted
    from memory, lookups still see them (stat) and loads read them back"""
    case = dict(CASE, chunks=6, num_blocks=128)
    root = disk_cache(3)
    src = HostKV(case)
    w = src.worker()
    w.register()
    bids = gen.block_ids(case)
    keys = keys_for(6, seed=2)
    for c in range(3):
        assert w.store(keys[2 * c:2 * c + 2], bids[2 * c * BPC:(2 * c + 2) * BPC]) == 0
    w.flush()
    st = w.stats()
    assert st["evictions"] == 3 and st["disk_writes"] == 6
    assert len(os.listdir(ns_dir(root))) == 6
    assert w.lookup(keys) == 6 * 32
    assert w.stats()["disk_lookup_hits"] == 3
    assert w.lookup_batch([keys, keys[:2], [b"\x01" * 32] + keys]).tolist() == [6, 2, 0]

    # memory now holds keys 3..5; load 0 and 1 (files) and 5 (memory) into a
    # zeroed cache registered under the same (model, tp) entry
    dst = HostKV(case, zero=True)
    w2 = dst.worker()
    w2.register()
    dst_bids = gen.block_ids(case, seed_offset=1)
    sel = [0, 1, 5]
    lk = [keys[i] for i in sel]
    lb = np.concatenate([bids[i * BPC:(i + 1) * BPC] for i in sel])
    db = np.concatenate([dst_bids[i * BPC:(i + 1) * BPC] for i in sel])
    assert w2.load(lk, db) == 0
    st = w2.stats()
    assert st["disk_reads"] == 2 and st["loaded"] == 3 and st["bytes_read_disk"] == 2 * REC
    k0, v0 = expected_scatter(src, lb, db)
    assert all(np.array_equal(a, b) for a, b in zip(dst.k, k0))
    assert all(np.array_equal(a, b) for a, b in zip(dst.v, v0))
    # the records read stay in memory: loading them again reads no file
    dst2 = HostKV(case, zero=True)
    w3 = dst2.worker()
    w3.register()
    assert w3.load(lk, db) == 0
    assert w3.stats()["disk_reads"] == 2
    assert all(np.array_equal(a, b) for a, b in zip(dst2.k, k0))
    for x in (w, w2, w3):
        x.unregister()


def test_persistence_across_restart(tmp_path):
    root = tmp_path / "persist"
    src = HostKV(CASE)
    bids = gen.block_ids(CASE)
    keys = keys_for(CASE["chunks"], seed=3)
    cc.init(CASE["chunk_size"], 4 * REC, str(root), CACHE_BACKEND_MEM)
    try:
        w = src.worker()
        w.register()
        assert w.store(keys, bids) == 0
    finally:
        cc.exit()                          # drains the write-behind
    assert len(os.listdir(ns_dir(root))) == CASE["chunks"]

    cc.init(CASE["chunk_size"], 4 * REC, str(root), CACHE_BACKEND_MEM)
    try:
        dst = HostKV(CASE, zero=True)
        w = dst.worker()
        w.register()
        assert w.lookup(keys) == len(keys) * 32
        dst_bids = gen.block_ids(CASE, seed_offset=1)
        assert w.load(keys, dst_bids) == 0
        k0, v0 = expected_scatter(src, bids, dst_bids)
        assert all(np.array_equal(a, b) for a, b in zip(dst.k, k0))
        assert all(np.array_equal(a, b) for a, b in zip(dst.v, v0))
        st = w.stats()
        assert st["disk_reads"] == CASE["chunks"] and st["stored"] == 0
        w.unregister()
    finally:
        cc.exit()


def test_missing_and_damaged_files(disk_cache):
    root = disk_cache(4)
    src = HostKV(CASE)
    w = src.worker()
    w.register()
    bids = gen.block_ids(CASE)
    keys = keys_for(3, seed=4)
    assert w.store(keys, bids) == 0
    w.clear()                              # waits for the files, empties memory
    assert w.stats()["records_used"] == 0
    (ns_dir(root) / keys[1].hex()).unlink()
    with open(ns_dir(root) / keys[2].hex(), "r+b") as f:
        f.truncate(REC - 4096)             # a record of the wrong size is no record
    assert w.lookup(keys) == 32
    assert w.lookup([keys[2]]) == 0
    dst = HostKV(CASE, zero=True)
    w2 = dst.worker()
    w2.register()
    dst_bids = gen.block_ids(CASE, seed_offset=1)
    assert w2.load(keys, dst_bids) == -errno.ENOENT
    st = w2.stats()
    assert st["disk_reads"] == 1 and st["load_misses"] == 2 and st["records_used"] == 1
    # the record that existed was still loaded
    k0, v0 = expected_scatter(src, bids[:BPC], dst_bids[:BPC])
    assert all(np.array_equal(a, b) for a, b in zip(dst.k, k0))
    w2.unregister()
    w.unregister()


def test_tp_ranks_keep_separate_files(disk_cache):
    """two ranks store different head shards under the same keys; each loads
    its own back (the reference's flat directory would mix them)"""
    root = disk_cache(4)
    keys = keys_for(CASE["chunks"], seed=5)
    bids = gen.block_ids(CASE)
    srcs, ws = [], []
    for r in range(2):
        s = HostKV(CASE, seed=100 + r)
        w = s.worker(world_size=2, rank=r)
        w.register()
        assert w.store(keys, bids) == 0
        w.clear()
        srcs.append(s)
        ws.append(w)
    assert sorted(os.listdir(root)) == ["m.tp2.0", "m.tp2.1"]
    dst_bids = gen.block_ids(CASE, seed_offset=1)
    for r in range(2):
        dst = HostKV(CASE, zero=True)
        w = dst.worker(world_size=2, rank=r)
        w.register()
        assert w.load(keys, dst_bids) == 0
        k0, v0 = expected_scatter(srcs[r], bids, dst_bids)
        assert all(np.array_equal(a, b) for a, b in zip(dst.k, k0))
        w.unregister()
    for w in ws:
        w.unregister()


def test_existing_file_is_not_rewritten(disk_cache):
    disk_cache(4)
    src = HostKV(CASE)
    w = src.worker()
    w.register()
    keys = keys_for(1, seed=6)
    bids = gen.block_ids(CASE)[:BPC]
    assert w.store(keys, bids) == 0
    w.clear()
    assert w.store(keys, bids) == 0        # memory miss, file present
    w.flush()
    st = w.stats()
    assert st["disk_writes"] == 1 and st["disk_write_skips"] == 1 and st["stored"] == 2
    w.unregister()


def test_model_tag_is_sanitised(disk_cache):
    root = disk_cache(2)
    src = HostKV(CASE)
    w = src.worker(name="meta-llama/Meta-Llama-3-8B")
    w.register()
    assert w.store(keys_for(1, seed=7), gen.block_ids(CASE)[:BPC]) == 0
    w.flush()
    assert os.listdir(root) == ["meta-llama_Meta-Llama-3-8B.tp1.0"]
    w.unregister()


def test_unusable_root_dir(tmp_path):
    f = tmp_path / "file"
    f.write_bytes(b"x")
    with pytest.raises(cc.CacheError) as e:
        cc.init(256, 1 << 20, str(f), CACHE_BACKEND_MEM)
    assert e.value.ret == -errno.ENOTDIR
    # a failed init leaves the manager uninitialised: a memory-only init works
    cc.init(256, 1 << 20, None, CACHE_BACKEND_MEM)
    cc.exit()


def test_flush_without_disk_tier():
    cc.init(CASE["chunk_size"], 2 * REC, None, CACHE_BACKEND_MEM)
    try:
        w = HostKV(CASE).worker()
        w.register()
        w.flush()
        assert w.stats()["disk_writes"] == 0
        w.unregister()
    finally:
        cc.exit()


def test_threads_store_and_reload_through_disk(disk_cache):
    """4 threads store their own records into a pool of 8 and reload older
    ones (mostly evicted to disk) into zeroed caches at the same blocks:
    every reloaded block equals its source block"""
    import threading

    case = dict(CASE, num_blocks=128, chunks=8)
    disk_cache(8)
    errors, reads = [], []

    def run(t):
        try:
            rng = np.random.default_rng(300 + t)
            src = HostKV(case, seed=200 + t)
            w = src.worker()
            w.register()
            keys = keys_for(8, seed=400 + t)
            bids = gen.block_ids(case)
            for it in range(12):
                c = it % 8
                assert w.store(keys[c:c + 1], bids[c * BPC:(c + 1) * BPC]) == 0
                j = int(rng.integers(0, c + 1)) if it < 8 else int(rng.integers(0, 8))
                dst = HostKV(case, zero=True)
                wd = dst.worker()
                wd.register()
                sel = bids[j * BPC:(j + 1) * BPC].astype(np.int64)
                ret = wd.load(keys[j:j + 1], sel)
                assert ret == 0, ret
                for a, b in zip(dst.k + dst.v, src.k + src.v):
                    blk = a.reshape(case["num_blocks"], -1)
                    ref = b.reshape(case["num_blocks"], -1)
                    assert np.array_equal(blk[sel], ref[sel])
                wd.unregister()
            w.flush()
            reads.append(w.stats()["disk_reads"])
            w.unregister()
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append((t, repr(e)))

    ths = [threading.Thread(target=run, args=(t,)) for t in range(4)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    assert not errors, errors
    assert max(reads) > 0          # the reloads did go through files
