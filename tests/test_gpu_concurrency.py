"""Thread safety and deadlines of the CUDA backend.

The reference calls transfer_kvcache from its 4 CaCopy threads at once
(src/cache/cache.c:777); stores and loads also run concurrently from the
server's store and load pools.  The deadline test makes the host-side wait
run out on a transfer that is merely slower than a 1 ms deadline: the device
work completes on its own afterwards, nothing hangs, and the next call on a
fresh lane succeeds."""
import ctypes as C
import errno
import threading

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from demo_b200._lib import TransferBatch, lib
from tests.golden import gen
from tests.gpu_util import DeviceKV

pytestmark = pytest.mark.gpu


def test_concurrent_stores_and_loads_from_threads():
    case = dict(num_blocks=2048, block_size=16, chunk_size=256, num_layers=4, hidden=1024, elt=2,
                kv=2, chunks=1, seed=21)
    src, dst = DeviceKV(case), DeviceKV(case, zero=True)
    rb = gen.record_bytes(case)
    cc.init(256, 80 * rb, None)
    try:
        lay = cc.KVLayout(4, 2048, 16, 1024, 2, 2)
        ws = cc.Worker("conc", lay, [t.data_ptr() for t in src.k], [t.data_ptr() for t in src.v])
        wd = cc.Worker("conc", lay, [t.data_ptr() for t in dst.k], [t.data_ptr() for t in dst.v])
        ws.register()
        wd.register()
        rng = np.random.default_rng(0)
        perm_s = rng.permutation(2048)
        perm_d = rng.permutation(2048)
        nthreads, per = 8, 8                       # 8 threads x 8 records
        keys = [[rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(per)] for _ in range(nthreads)]
        rets = {}

        def worker(i):
            bs = perm_s[i * per * 16:(i + 1) * per * 16].astype(np.uint64)
            bd = perm_d[i * per * 16:(i + 1) * per * 16].astype(np.uint64)
            r1 = ws.store(keys[i], bs)
            r2 = wd.load(keys[i], bd)
            rets[i] = (r1, r2)

        th = [threading.Thread(target=worker, args=(i,)) for i in range(nthreads)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert all(v == (0, 0) for v in rets.values()), rets
        n = nthreads * per * 16
        s_idx = torch.from_numpy(perm_s[:n].astype(np.int64)).cuda()
        d_idx = torch.from_numpy(perm_d[:n].astype(np.int64)).cuda()
        blk = 16 * 2048
        for a, b in zip(src.k + src.v, dst.k + dst.v):
            assert torch.equal(a.view(-1, blk)[s_idx], b.view(-1, blk)[d_idx])
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()


def test_host_deadline_returns_etimedout_and_context_stays_usable(monkeypatch):
    case = dict(num_blocks=4096, block_size=16, chunk_size=256, num_layers=8, hidden=1024, elt=2,
                kv=2, chunks=64, seed=22)
    kv = DeviceKV(case)
    rb = gen.record_bytes(case)                   # 8 MiB records, 512 MiB per call
    n = case["chunks"]
    bids = gen.block_ids(case)

    def batch(ad):
        daddr = C.c_void_p()
        host = lib.alloc_pinned_ptr(ad, 0, n * rb, 0, C.byref(daddr))
        assert host
        kp = np.array([t.data_ptr() for t in kv.k], np.uint64)
        vp = np.array([t.data_ptr() for t in kv.v], np.uint64)
        dk = lib.open_ipc_keys(ad, 0, 8, len(kp), kp.ctypes.data)
        dv = lib.open_ipc_keys(ad, 0, 8, len(vp), vp.ctypes.data)
        arr = (C.c_void_p * n)(*[host + i * rb for i in range(n)])
        b = np.ascontiguousarray(bids)
        tb = TransferBatch(keys_ptrs=dk, value_ptrs=dv, page_buffer_size=4096 * 16, records=arr,
                           block_ids=b.ctypes.data_as(C.POINTER(C.c_uint64)), num_records=n, block_size=16,
                           hidden_dim_size=1024, num_layers=8, num_tokens=256, devid=0,
                           caches_element_size=2, record_on_device=0, direction=True)
        return lib.transfer_kvcache_batch(ad, C.byref(tb)), host

    monkeypatch.setenv("CROSSCACHE_TIMEOUT_MS", "1")      # 512 MiB over PCIe takes ~10 ms
    slow = lib.cuda_adaptor_create()
    ret, host1 = batch(slow)
    assert ret == -errno.ETIMEDOUT
    torch.cuda.synchronize()                               # the device finishes the work by itself
    monkeypatch.setenv("CROSSCACHE_TIMEOUT_MS", "120000")
    ok = lib.cuda_adaptor_create()
    ret, host2 = batch(ok)
    assert ret == 0
    got = np.ctypeslib.as_array((C.c_uint8 * rb).from_address(host2))
    k, v = gen.paged_layers(case)
    from oracle import kvcopy as okc
    exp = okc.gather(k, v, bids[:16], 256, 16, 2048)[0]
    assert np.array_equal(got, exp)
    lib.cuda_adaptor_destroy(ok)
    lib.cuda_adaptor_destroy(slow)
