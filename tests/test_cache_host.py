"""Cache-manager host logic through the public C API on the explicit CPU
(MEM) backend: chunking, record layout, dedupe, lookup semantics, LRU
eviction, errors.  Paged layers are numpy arrays; the oracle checks bytes."""
import ctypes as C
import errno
import os

import numpy as np
import pytest

from demo_b200 import cache as cc
from demo_b200._lib import CACHE_BACKEND_MEM, TransferParams, lib
from oracle import blockhash as bh
from oracle import kvcopy as ok
from oracle.cache_model import LRUPool
from tests.golden import gen


def keys_for(n, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(n)]


class HostKV:
    def __init__(self, case, seed=None, zero=False):
        self.case = case
        self.k, self.v = gen.paged_layers(case, seed=seed, zero=zero)
        self.layout = cc.KVLayout(case["num_layers"], case["num_blocks"], case["block_size"],
                                  case["hidden"], case["elt"], case["kv"])

    def worker(self, name="m", world_size=1, rank=0):
        return cc.Worker(name, self.layout, [a.ctypes.data for a in self.k],
                         [a.ctypes.data for a in self.v] if self.v is not None else None,
                         node_id=0, world_size=world_size, rank=rank)


@pytest.fixture
def mem_cache():
    def _init(records, case, chunk=None):
        cc.init(chunk or case["chunk_size"], records * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    yield _init
    cc.exit()


CACHE_CASES = [c for c in gen.KV_CASES if gen.record_bytes(c) % 4096 == 0]


def test_register_rejects_records_not_4k_aligned(mem_cache):
    """reference cache.c:621-622 asserts chunk bytes % 4096 == 0"""
    case = next(c for c in gen.KV_CASES if gen.record_bytes(c) % 4096)
    mem_cache(4, case)
    with pytest.raises(cc.CacheError) as e:
        HostKV(case).worker().register()
    assert e.value.ret == -errno.EINVAL


@pytest.mark.parametrize("case", CACHE_CASES, ids=lambda c: c["name"])
def test_store_load_roundtrip_matches_oracle(case, mem_cache):
    mem_cache(case["chunks"] + 1, case)
    src = HostKV(case)
    w = src.worker()
    w.register()
    bids = gen.block_ids(case)
    keys = keys_for(case["chunks"])
    assert w.store(keys, bids) == 0
    st = w.stats()
    assert st["stored"] == case["chunks"] and st["records_used"] == case["chunks"]
    w.unregister()

    # reload into a second, zeroed cache at a fresh block table
    dst = HostKV(case, zero=True)
    w2 = dst.worker()
    mem_cache_entries = None  # same (model, tp) entry survives? no: unregister freed it
    del mem_cache_entries
    cc.exit()
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    w1 = src.worker()
    w1.register()
    assert w1.store(keys, bids) == 0
    w2 = dst.worker(name="m")            # same model/tp: shares the entry (ref 2)
    w2.register()
    bids2 = gen.block_ids(case, seed_offset=1)
    assert w2.load(keys, bids2) == 0
    exp_k, exp_v = gen.paged_layers(case, zero=True)
    recs = ok.gather(src.k, src.v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    ok.scatter(recs, exp_k, exp_v, bids2, case["chunk_size"], case["block_size"], gen.unit_of(case))
    for a, b in zip(dst.k, exp_k):
        assert np.array_equal(a, b)
    if dst.v is not None:
        for a, b in zip(dst.v, exp_v):
            assert np.array_equal(a, b)
    w2.unregister()
    w1.unregister()


def test_c1_cpu_plumbing_llama2_7b(mem_cache):
    """Llama-2-7B KV (32 layers, 32 heads x 128, fp16, block 16),
    256 blocks = 16 chunks of 256 tokens; KV ~ N(0,1) fp16 seed 0, tokens
    U[0,32000) seed 1, keys = chained vLLM sha256 block hashes strided every
    16 blocks.  Put all 256 blocks, get them back into a fresh block table,
    verify byte equality and key identity."""
    import torch

    L, H, D, bs, nb = 32, 32, 128, 16, 256
    unit = H * D * 2
    case = dict(num_blocks=nb, block_size=bs, chunk_size=256, num_layers=L, hidden=H * D, elt=2,
                kv=2, chunks=16, seed=0)
    g = torch.Generator().manual_seed(0)
    k = [torch.randn(nb * bs * H * D, generator=g).half().numpy().view(np.uint8) for _ in range(L)]
    v = [torch.randn(nb * bs * H * D, generator=g).half().numpy().view(np.uint8) for _ in range(L)]
    tokens = torch.randint(0, 32000, (nb * bs,), generator=torch.Generator().manual_seed(1)).tolist()
    hashes = bh.block_hashes(tokens, bs, bh.none_hash("0"))
    keys = bh.chunk_keys(hashes, 256 // bs)
    assert len(keys) == 16
    mem_cache(16, case)
    lay = cc.KVLayout(L, nb, bs, H * D, 2, 2)
    w = cc.Worker("llama-2-7b", lay, [a.ctypes.data for a in k], [a.ctypes.data for a in v])
    w.register()
    bids = np.random.default_rng(2).permutation(nb).astype(np.uint64)
    assert w.store(keys, bids) == 0
    assert w.lookup(keys) == 16 * 32
    w.unregister()
    k2 = [np.zeros_like(a) for a in k]
    v2 = [np.zeros_like(a) for a in v]
    # same entry (model, tp) still registered? no -> store again through a
    # worker on the original cache, then load into the fresh one
    w = cc.Worker("llama-2-7b", lay, [a.ctypes.data for a in k], [a.ctypes.data for a in v])
    w.register()
    assert w.store(keys, bids) == 0
    wd = cc.Worker("llama-2-7b", lay, [a.ctypes.data for a in k2], [a.ctypes.data for a in v2])
    wd.register()
    bids2 = np.random.default_rng(3).permutation(nb).astype(np.uint64)
    assert wd.load(keys, bids2) == 0
    # byte equality: block bids[i] of the source == block bids2[i] of the destination
    blk = bs * unit
    for l in range(L):
        src = k[l].reshape(nb, blk)[bids.astype(np.int64)]
        dst = k2[l].reshape(nb, blk)[bids2.astype(np.int64)]
        assert np.array_equal(src, dst)
        src = v[l].reshape(nb, blk)[bids.astype(np.int64)]
        dst = v2[l].reshape(nb, blk)[bids2.astype(np.int64)]
        assert np.array_equal(src, dst)
    assert wd.stats()["loaded"] == 16
    wd.unregister()
    w.unregister()


def test_lookup_returns_byte_offset_of_first_miss(mem_cache):
    case = gen.KV_CASES[0]
    mem_cache(8, case)
    kv = HostKV(case)
    w = kv.worker()
    w.register()
    keys = keys_for(4, seed=5)
    bpc = case["chunk_size"] // case["block_size"]
    assert w.store(keys[:2], np.arange(2 * bpc)) == 0
    assert w.lookup(keys) == 2 * 32
    assert w.lookup(keys[2:]) == 0
    assert w.lookup([keys[0], keys[3], keys[1]]) == 32      # stops at the first miss
    assert w.lookup([]) == 0
    other = kv.worker(name="unregistered")
    assert other.lookup(keys) == 0                           # unknown model -> 0 (cache.c:725-727)
    assert list(w.lookup_batch([keys, keys[1:], keys[3:], []])) == [2, 1, 0, 0]
    w.unregister()


def test_store_dedupes_existing_keys_and_keeps_first_record(mem_cache):
    case = gen.KV_CASES[0]
    mem_cache(8, case)
    kv = HostKV(case)
    w = kv.worker()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    key = keys_for(1, seed=9)
    b1 = np.arange(bpc, dtype=np.uint64)
    b2 = np.arange(bpc, 2 * bpc, dtype=np.uint64)
    assert w.store(key, b1) == 0
    assert w.store(key, b2) == 0                  # same key: existing record kept
    assert w.store(key + key, np.concatenate([b2, b2])) == 0   # in-batch duplicate
    st = w.stats()
    assert st["stored"] == 1 and st["store_dedup"] == 3
    w.unregister()
    cc.exit()
    # what a load returns is the FIRST stored content (blocks b1)
    cc.init(case["chunk_size"], 8 * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    w = kv.worker()
    w.register()
    assert w.store(key, b1) == 0
    assert w.store(key, b2) == 0
    dst = HostKV(case, zero=True)
    wd = dst.worker()
    wd.register()
    assert wd.load(key, b2) == 0
    exp_k, exp_v = gen.paged_layers(case, zero=True)
    ok.scatter(ok.gather(kv.k, kv.v, b1, case["chunk_size"], case["block_size"], gen.unit_of(case)),
               exp_k, exp_v, b2, case["chunk_size"], case["block_size"], gen.unit_of(case))
    assert all(np.array_equal(a, b) for a, b in zip(dst.k, exp_k))
    wd.unregister()
    w.unregister()


def test_lru_eviction_matches_model(mem_cache):
    case = gen.KV_CASES[0]
    cap = 4
    mem_cache(cap, case)
    kv = HostKV(case)
    w = kv.worker()
    w.register()
    model = LRUPool(cap)
    bpc = case["chunk_size"] // case["block_size"]
    keys = keys_for(10, seed=21)
    rng = np.random.default_rng(4)
    for step in range(60):
        op = rng.integers(0, 3)
        sel = [keys[i] for i in rng.choice(10, size=int(rng.integers(1, 4)), replace=False)]
        if op == 0:
            assert w.store(sel, np.zeros(bpc * len(sel), np.uint64)) == 0
            model.store(sel)
        elif op == 1:
            assert w.lookup(sel) // 32 == model.lookup(sel)
        else:
            hits = model.load(sel)
            ret = w.load(sel, np.zeros(bpc * len(sel), np.uint64))
            assert ret == (0 if all(hits) else -errno.ENOENT)
        st = w.stats()
        assert st["evictions"] == model.evictions, step
        assert st["records_used"] == len(model.od)
    w.unregister()


def test_load_of_missing_key_fails_but_loads_the_hits(mem_cache):
    case = gen.KV_CASES[1]
    mem_cache(4, case)
    src = HostKV(case)
    w = src.worker()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    keys = keys_for(2, seed=33)
    bids = gen.block_ids(case)[: 2 * bpc]
    assert w.store(keys[:1], bids[:bpc]) == 0
    dst = HostKV(case, zero=True)
    wd = dst.worker(name="m")
    wd.register()
    assert wd.load([keys[0], keys[1]], bids) == -errno.ENOENT
    st = wd.stats()
    assert st["loaded"] == 1 and st["load_misses"] == 1
    blk = case["block_size"] * gen.unit_of(case)
    for l in range(case["num_layers"]):
        a = src.k[l].reshape(-1, blk)[bids[:bpc].astype(np.int64)]
        b = dst.k[l].reshape(-1, blk)[bids[:bpc].astype(np.int64)]
        assert np.array_equal(a, b)
        assert not dst.k[l].reshape(-1, blk)[bids[bpc:].astype(np.int64)].any()
    wd.unregister()
    w.unregister()


def test_pool_exhaustion_and_partial_chunks(mem_cache):
    case = gen.KV_CASES[0]
    mem_cache(2, case)
    kv = HostKV(case)          # owns the paged layers for the life of the worker
    w = kv.worker()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    keys = keys_for(3, seed=44)
    # one call needing more records than the pool holds: the records of this
    # call are all in flight, nothing is evictable -> -ENOMEM for the rest
    # (the reference spins forever here, cache.c:329-335)
    assert w.store(keys, np.arange(3 * bpc)) == -errno.ENOMEM
    assert w.lookup(keys) == 2 * 32
    # a later call recycles the least-recently-used record
    k3 = keys_for(1, seed=47)
    assert w.store(k3, np.arange(bpc)) == 0
    assert w.stats()["evictions"] == 1
    assert w.lookup(keys[:1]) == 0 and w.lookup(keys[1:2] + k3) == 2 * 32
    # bnum not a multiple of the chunk: trailing blocks are ignored (integer division)
    assert w.store(keys_for(1, seed=45), np.arange(bpc + 1)) == 0
    assert w.store(keys_for(1, seed=46), np.arange(bpc - 1)) == 0    # zero chunks
    w.unregister()


def test_errors(mem_cache):
    case = gen.KV_CASES[0]
    mem_cache(4, case)
    kv = HostKV(case)
    w = kv.worker()
    assert w.store(keys_for(1), np.arange(2)) == -errno.ENOENT     # not registered
    bad = kv.worker()
    bad.ctx.per_token_size += 2
    with pytest.raises(cc.CacheError):
        bad.register()
    ipc = kv.worker()
    ipc.ctx.per_len = 64        # MEM backend takes raw host pointers only
    with pytest.raises(cc.CacheError):
        ipc.register()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    # a block id outside the paged cache: -EINVAL, nothing published
    bids = np.array([case["num_blocks"]] + [0] * (bpc - 1), dtype=np.uint64)
    k1 = keys_for(1, seed=77)
    assert w.store(k1, bids) == -errno.EINVAL
    assert w.lookup(k1) == 0
    kb = b"".join(k1)
    assert lib.cache_store(C.byref(w.ctx), kb, 16, np.zeros(bpc, np.uint64).ctypes.data, bpc) == -errno.EINVAL
    assert cc.lib.cache_init_backend(256, 1 << 20, None, CACHE_BACKEND_MEM) == -errno.EBUSY
    w.unregister()


def test_clear_and_stats(mem_cache):
    case = gen.KV_CASES[0]
    mem_cache(4, case)
    kv = HostKV(case)          # owns the paged layers for the life of the worker
    w = kv.worker()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    keys = keys_for(3, seed=55)
    assert w.store(keys, np.arange(3 * bpc)) == 0
    assert w.stats()["records_used"] == 3
    w.clear()
    assert w.stats()["records_used"] == 0
    assert w.lookup(keys) == 0
    st = w.stats()
    assert st["records_total"] == 4 and st["bytes_saved"] == 3 * gen.record_bytes(case)
    w.unregister()


@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_per_chunk_transfer_abi_mem_adaptor(case):
    """transfer_kvcache with a reference-style slot mapping (wrapper_ptr)."""
    ad = lib.mem_adaptor_create()
    try:
        k, v = gen.paged_layers(case)
        kp = np.array([a.ctypes.data for a in k], np.uint64)
        vp = np.array([a.ctypes.data for a in v], np.uint64) if v is not None else None
        dk = lib.open_ipc_keys(ad, 0, 8, len(kp), kp.ctypes.data)
        dv = lib.open_ipc_keys(ad, 0, 8, len(vp), vp.ctypes.data) if v is not None else None
        bids = gen.block_ids(case)
        bpc = case["chunk_size"] // case["block_size"]
        slots = ok.slot_mapping(bids[:bpc], case["block_size"])
        dslots = lib.wrapper_ptr(ad, 0, slots.ctypes.data, slots.nbytes)
        rec = np.zeros(gen.record_bytes(case), np.uint8)
        p = TransferParams(caches=rec.ctypes.data, caches_h=rec.ctypes.data, keys_ptrs=dk, value_ptrs=dv,
                           page_buffer_size=case["num_blocks"] * case["block_size"], slot_mapping=dslots,
                           devid=0, caches_element_size=case["elt"], num_layers=case["num_layers"],
                           num_tokens=case["chunk_size"], hidden_dim_size=case["hidden"], direction=True)
        assert lib.transfer_kvcache(ad, C.byref(p)) == 0
        exp = ok.gather(k, v, bids[:bpc], case["chunk_size"], case["block_size"], gen.unit_of(case))[0]
        assert np.array_equal(rec, exp)
        lib.unwrapper_ptr(ad, dslots)
        lib.close_ipc_keys(ad, dk)
        if dv:
            lib.close_ipc_keys(ad, dv)
    finally:
        lib.mem_adaptor_destroy(ad)


def test_key_stride_wider_than_32_bytes_and_empty_calls(mem_cache):
    """keys are compared on their first 32 bytes at a key_len stride
    (reference cache.c:139-145,538-546); empty calls are no-ops"""
    case = gen.KV_CASES[0]
    mem_cache(8, case)
    kv = HostKV(case)          # owns the paged layers for the life of the worker
    w = kv.worker()
    w.register()
    bpc = case["chunk_size"] // case["block_size"]
    k = keys_for(3, seed=90)
    stride = 48
    buf = b"".join(x + bytes([7]) * (stride - 32) for x in k)
    bids = np.arange(3 * bpc, dtype=np.uint64)
    assert cc.lib.cache_store(C.byref(w.ctx), buf, stride, bids.ctypes.data, len(bids)) == 0
    assert cc.lib.cache_lookup(C.byref(w.ctx), buf, 3, stride) == 3 * stride
    # the padding bytes are not part of the key
    buf2 = b"".join(x + bytes([9]) * (stride - 32) for x in k)
    assert cc.lib.cache_lookup(C.byref(w.ctx), buf2, 3, stride) == 3 * stride
    assert w.lookup(k) == 3 * 32
    assert cc.lib.cache_store(C.byref(w.ctx), buf, stride, bids.ctypes.data, 0) == 0
    assert cc.lib.cache_load(C.byref(w.ctx), buf, stride, bids.ctypes.data, 0) == 0
    assert cc.lib.cache_lookup(C.byref(w.ctx), buf, 0, stride) == 0
    w.unregister()


def test_batch_entry_points_report_per_request(mem_cache):
    """cache_store_batch / cache_load_batch: one transfer, a result per
    request -- a request with a missing key fails alone"""
    case = next(c for c in CACHE_CASES if c["name"] == "gqa_bs16")
    case = dict(case, chunks=6, num_blocks=128)
    bpc = case["chunk_size"] // case["block_size"]
    mem_cache(8, case)
    src, dst = HostKV(case), HostKV(case, zero=True)
    ws, wd = src.worker(), dst.worker()
    ws.register()
    wd.register()
    keys = keys_for(6, seed=51)
    bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
    split = [(0, 2), (2, 3), (3, 6)]
    kreq = [keys[a:b] for a, b in split]
    breq = [bids[a * bpc:b * bpc] for a, b in split]
    ret, st = ws.store_batch(kreq, breq)
    assert ret == 0 and st.tolist() == [0, 0, 0]
    assert ws.stats()["stored"] == 6
    # request 1 asks for a key that was never stored
    missing = keys_for(1, seed=52)
    lreq = [keys[0:2], missing + keys[2:3], keys[3:6]]
    lb = [b2[0:2 * bpc], b2[2 * bpc:4 * bpc], b2[4 * bpc:7 * bpc]] if len(b2) >= 7 * bpc else None
    if lb is None:
        b2 = np.random.default_rng(5).permutation(case["num_blocks"])[:7 * bpc].astype(np.uint64)
        lb = [b2[0:2 * bpc], b2[2 * bpc:4 * bpc], b2[4 * bpc:7 * bpc]]
    ret, st = wd.load_batch(lreq, lb)
    assert ret == -errno.ENOENT
    assert st.tolist() == [0, -errno.ENOENT, 0]
    # every cached key was still loaded where it was asked for
    src_sel = np.concatenate([bids[0:2 * bpc], bids[2 * bpc:3 * bpc], bids[3 * bpc:6 * bpc]])
    dst_sel = np.concatenate([lb[0], lb[1][bpc:], lb[2]])
    recs = ok.gather(src.k, src.v, src_sel, case["chunk_size"], case["block_size"], gen.unit_of(case))
    ek, ev = gen.paged_layers(case, zero=True)
    ok.scatter(recs, ek, ev, dst_sel, case["chunk_size"], case["block_size"], gen.unit_of(case))
    assert all(np.array_equal(a, b) for a, b in zip(dst.k, ek))
    assert all(np.array_equal(a, b) for a, b in zip(dst.v, ev))
    # more new keys in one call than the pool has records (8): the keys past
    # that point fail, and only the request that holds them
    more = keys_for(10, seed=53)
    blk = np.tile(bids[:bpc], 10)
    ret, st = ws.store_batch([more[:6], more[6:]], [blk[:6 * bpc], blk[6 * bpc:]])
    assert ret == -errno.ENOMEM and st.tolist() == [0, -errno.ENOMEM]
    with pytest.raises(ValueError):
        ws.store_batch([keys[:1]], [bids[:bpc - 1]])
    wd.unregister()
    ws.unregister()
