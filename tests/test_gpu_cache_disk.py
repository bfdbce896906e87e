"""Disk tier on the CUDA backend: records saved from device paged caches are
written to files with the reference's record bytes, and come back bit-exact
after eviction and after a cache restart (HBM -> pinned host -> file ->
pinned host -> HBM)."""
import hashlib
import os

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from oracle import kvcopy as ok
from tests.golden import gen
from tests.gpu_util import DeviceKV
from tests.test_gpu_cache import keys_for, worker

pytestmark = pytest.mark.gpu

CASES = [c for c in gen.KV_CASES if gen.record_bytes(c) % 4096 == 0]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_files_then_restart_then_load(case, tmp_path, golden_records):
    root = tmp_path / "kv"
    keys = keys_for(case["chunks"], seed=11)
    bids, bids2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
    rec = gen.record_bytes(case)

    cc.init(case["chunk_size"], (case["chunks"] + 1) * rec, str(root))
    try:
        src = DeviceKV(case)
        w = worker(src)
        w.register()
        assert w.store(keys, bids) == 0
        w.flush()
        assert w.stats()["disk_writes"] == case["chunks"]
        g = golden_records[case["name"]]
        for k, digest in zip(keys, g["record_sha256"]):
            assert hashlib.sha256((root / "m.tp1.0" / k.hex()).read_bytes()).hexdigest() == digest
        w.unregister()
    finally:
        cc.exit()

    cc.init(case["chunk_size"], (case["chunks"] + 1) * rec, str(root))
    try:
        dst = DeviceKV(case, zero=True)
        w = worker(dst)
        w.register()
        assert w.lookup(keys) == 32 * case["chunks"]
        assert w.load(keys, bids2) == 0
        torch.cuda.synchronize()
        k, v = gen.paged_layers(case)
        ek, ev = gen.paged_layers(case, zero=True)
        recs = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
        ok.scatter(recs, ek, ev, bids2, case["chunk_size"], case["block_size"], gen.unit_of(case))
        kh, vh = dst.host()
        assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
        if vh is not None:
            assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
        st = w.stats()
        assert st["disk_reads"] == case["chunks"] and st["loaded"] == case["chunks"]
        w.unregister()
    finally:
        cc.exit()


def test_eviction_to_disk_and_mixed_load(tmp_path):
    """a pool of 2 records under 4 stores; one load takes 1 memory record and
    1 file record in the same batched transfer"""
    case = dict(next(c for c in CASES if c["name"] == "tp8_shard"), chunks=4)
    rec = gen.record_bytes(case)
    bpc = case["chunk_size"] // case["block_size"]
    cc.init(case["chunk_size"], 2 * rec, str(tmp_path / "kv"))
    try:
        src, dst = DeviceKV(case), DeviceKV(case, zero=True)
        ws, wd = worker(src), worker(dst)
        ws.register()
        wd.register()
        keys = keys_for(4, seed=12)
        bids = gen.block_ids(case)
        for c in range(4):
            assert ws.store(keys[c:c + 1], bids[c * bpc:(c + 1) * bpc]) == 0
        ws.flush()
        assert ws.stats()["evictions"] == 2
        assert len(os.listdir(tmp_path / "kv" / "m.tp1.0")) == 4
        sel = [0, 3]                          # 0 on disk only, 3 in memory
        lb = np.concatenate([bids[i * bpc:(i + 1) * bpc] for i in sel])
        assert wd.load([keys[i] for i in sel], lb) == 0
        torch.cuda.synchronize()
        st = wd.stats()
        assert st["disk_reads"] == 1 and st["loaded"] == 2
        for a, b in zip(dst.k + dst.v, src.k + src.v):
            blk = a.view(case["num_blocks"], -1)[torch.as_tensor(lb.astype(np.int64), device="cuda")]
            ref = b.view(case["num_blocks"], -1)[torch.as_tensor(lb.astype(np.int64), device="cuda")]
            assert torch.equal(blk, ref)
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()
