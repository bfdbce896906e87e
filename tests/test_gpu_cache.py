"""Cache-manager C API on the CUDA backend: store/load round trips against the
oracle, lookup/dedupe/LRU semantics, the prefix-reuse workload shape, and
size-independent properties at larger sizes."""
import errno

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from demo_b200._lib import lib
from oracle import blockhash as bh
from oracle import kvcopy as ok
from oracle.cache_model import LRUPool
from tests.golden import gen
from tests.gpu_util import DeviceKV

pytestmark = pytest.mark.gpu

CACHE_CASES = [c for c in gen.KV_CASES if gen.record_bytes(c) % 4096 == 0]


def keys_for(n, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(n)]


def worker(kv: DeviceKV, name="m", world_size=1, rank=0):
    c = kv.case
    lay = cc.KVLayout(c["num_layers"], c["num_blocks"], c["block_size"], c["hidden"], c["elt"], c["kv"])
    return cc.Worker(name, lay, [t.data_ptr() for t in kv.k],
                     [t.data_ptr() for t in kv.v] if kv.v is not None else None,
                     node_id=torch.cuda.current_device(), world_size=world_size, rank=rank)


@pytest.fixture
def cuda_cache():
    def _init(records, case):
        cc.init(case["chunk_size"], records * gen.record_bytes(case), None)
    yield _init
    cc.exit()


@pytest.mark.parametrize("case", CACHE_CASES, ids=lambda c: c["name"])
def test_store_then_load_into_fresh_block_table(case, cuda_cache):
    cuda_cache(case["chunks"] + 2, case)
    src, dst = DeviceKV(case), DeviceKV(case, zero=True)
    ws, wd = worker(src), worker(dst)          # same (model, tp): one shared entry
    ws.register()
    wd.register()
    keys = keys_for(case["chunks"], seed=1)
    bids, bids2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
    launches = lib.crosscache_kernel_launches()
    assert ws.store(keys, bids) == 0
    assert ws.lookup(keys) == 32 * case["chunks"]
    assert wd.load(keys, bids2) == 0
    assert lib.crosscache_kernel_launches() > launches        # the CUDA kernels ran
    k, v = gen.paged_layers(case)
    ek, ev = gen.paged_layers(case, zero=True)
    recs = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    ok.scatter(recs, ek, ev, bids2, case["chunk_size"], case["block_size"], gen.unit_of(case))
    kh, vh = dst.host()
    assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
    if vh is not None:
        assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
    st = ws.stats()
    assert st["stored"] == case["chunks"] and st["loaded"] == case["chunks"]
    wd.unregister()
    ws.unregister()


def test_lru_dedupe_and_lookup_semantics_on_cuda_backend(cuda_cache):
    case = gen.KV_CASES[1]
    cap = 3
    cuda_cache(cap, case)
    kv = DeviceKV(case)
    w = worker(kv)
    w.register()
    model = LRUPool(cap)
    bpc = case["chunk_size"] // case["block_size"]
    keys = keys_for(6, seed=2)
    rng = np.random.default_rng(9)
    for step in range(40):
        op = int(rng.integers(0, 3))
        sel = [keys[i] for i in rng.choice(6, size=int(rng.integers(1, 3)), replace=False)]
        bids = rng.permutation(case["num_blocks"])[: bpc * len(sel)].astype(np.uint64)
        if op == 0:
            assert w.store(sel, bids) == 0
            model.store(sel)
        elif op == 1:
            assert w.lookup(sel) == 32 * model.lookup(sel)
        else:
            hits = model.load(sel)
            assert w.load(sel, bids) == (0 if all(hits) else -errno.ENOENT)
        assert w.stats()["evictions"] == model.evictions
    w.unregister()


def test_prefix_reuse_shape_hits_and_loads_only_hit_blocks(cuda_cache):
    """configs[2] scaled down: requests = shared prefix + unique suffix; save
    half, look up the other half: hits equal the shared-prefix chunks."""
    case = dict(num_blocks=1024, block_size=16, chunk_size=256, num_layers=4, hidden=1024, elt=2,
                kv=2, chunks=1, seed=5)
    cuda_cache(64, case)
    kv = DeviceKV(case)
    w = worker(kv)
    w.register()
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 128256, 1024).tolist()
    reqs = [prefix + rng.integers(0, 128256, 512).tolist() for _ in range(8)]
    nh = bh.none_hash("0")
    req_keys = [bh.chunk_keys(bh.block_hashes(t, 16, nh), 16) for t in reqs]
    assert all(len(k) == 6 for k in req_keys)
    perm = rng.permutation(case["num_blocks"])
    for i in range(4):
        assert w.store(req_keys[i], perm[i * 96:(i + 1) * 96].astype(np.uint64)) == 0
    st = w.stats()
    assert st["stored"] == 4 + 4 * 2 and st["store_dedup"] == 3 * 4     # prefix stored once
    hits = w.lookup_batch(req_keys[4:])
    assert hits.tolist() == [4, 4, 4, 4]                                  # 64 prefix blocks each
    for i in range(4, 8):
        n = int(hits[i - 4])
        assert w.load(req_keys[i][:n], perm[i * 96: i * 96 + n * 16].astype(np.uint64)) == 0
    # loaded prefix blocks equal the first request's prefix blocks
    k, v = kv.host()
    blk = 16 * 2048
    for l in range(4):
        a = k[l].reshape(-1, blk)
        for i in range(4, 8):
            assert np.array_equal(a[perm[i * 96: i * 96 + 64]], a[perm[0:64]])
    w.unregister()


def test_large_roundtrip_checksums():
    """Llama-3-8B layer shapes (8 heads x 128 bf16, block 16) with 2048
    blocks per layer and 32 layers: save 64 chunks, reload into a fresh
    block table; per-block checksums must match (size-independent check)."""
    L, nb, bs, H, D = 32, 2048, 16, 8, 128
    unit = H * D * 2
    g = torch.Generator(device="cuda").manual_seed(0)
    layers = [torch.randn(2, nb, bs, H, D, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
              for _ in range(L)]
    fresh = [torch.zeros_like(t) for t in layers]
    lay, kp, vp = cc.layout_from_kv_tensors(layers)
    assert lay.unit == unit and lay.kv == 2
    rec = lay.per_token_size * 256
    cc.init(256, 64 * rec, None)
    try:
        ws = cc.Worker("llama-3-8b", lay, kp, vp)
        _, kp2, vp2 = cc.layout_from_kv_tensors(fresh)
        wd = cc.Worker("llama-3-8b", lay, kp2, vp2)
        ws.register()
        wd.register()
        rng = np.random.default_rng(2)
        bids = rng.permutation(nb)[: 64 * 16].astype(np.uint64)
        bids2 = rng.permutation(nb)[: 64 * 16].astype(np.uint64)
        keys = keys_for(64, seed=3)
        assert ws.store(keys, bids) == 0
        assert wd.load(keys, bids2) == 0
        b1 = torch.from_numpy(bids.astype(np.int64)).cuda()
        b2 = torch.from_numpy(bids2.astype(np.int64)).cuda()
        for s, d in zip(layers, fresh):
            assert torch.equal(s[:, b1].view(torch.int16), d[:, b2].view(torch.int16))
        # untouched blocks of the destination stay zero
        mask = torch.ones(nb, dtype=torch.bool, device="cuda")
        mask[b2] = False
        assert all(int(d[:, mask].view(torch.int16).abs().sum()) == 0 for d in fresh)
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()
