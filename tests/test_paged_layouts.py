"""Paged layouts other than the reference's dense FlashAttention planes, on
the CPU (MEM) backend: vLLM FlashInfer's [num_blocks][2][...] blocks,
token-major (NHD) and head-major (HND, what vLLM uses on sm_100).  Layout
detection from tensor strides, register-time validation, and record bytes:
a FlashInfer cache holding the golden case's KV writes exactly the golden
records of the reference layout, and loads them back into its own layout."""
import ctypes as C
import errno
import hashlib

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from demo_b200 import protocol as P
from demo_b200._lib import CACHE_BACKEND_MEM, lib
from oracle import kvcopy as ok
from tests.flashinfer_layout import (as_flash_attn_view, as_vllm_view, from_flashinfer, head_bytes_of,
                                     to_flashinfer)
from tests.golden import gen
from tests.test_cache_host import keys_for

CASES = [c for c in gen.KV_CASES if c["kv"] == 2 and gen.record_bytes(c) % 4096 == 0]


def fi_tensors(case, hnd, zero=False):
    k, v = gen.paged_layers(case, zero=zero)
    phys = [torch.from_numpy(a) for a in to_flashinfer(case, k, v, hnd)]
    return phys, [as_vllm_view(case, p, hnd) for p in phys]


# ---- layout detection ----------------------------------------------------

@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
def test_flashinfer_geometry_from_strides(hnd):
    case = next(c for c in CASES if c["name"] == "gqa_bs16")
    unit, bs = gen.unit_of(case), case["block_size"]
    phys, views = fi_tensors(case, hnd)
    lay, kp, vp = cc.layout_from_kv_tensors(views)
    assert (lay.num_layers, lay.num_blocks, lay.block_size) == (case["num_layers"], case["num_blocks"], bs)
    assert lay.hidden_dim_size * lay.element_size == unit and lay.kv == 2
    assert lay.block_stride == 2 * bs * unit
    assert lay.head_bytes == (head_bytes_of(case) if hnd else 0)
    assert kp == [p.data_ptr() for p in phys]
    assert vp == [p.data_ptr() + bs * unit for p in phys]


def test_flash_attn_dense_and_head_major():
    case = next(c for c in CASES if c["name"] == "gqa_bs16")
    k, v = gen.paged_layers(case)
    unit, nb, bs = gen.unit_of(case), case["num_blocks"], case["block_size"]
    dense = [as_flash_attn_view(case, torch.from_numpy(a), torch.from_numpy(b)) for a, b in zip(k, v)]
    lay, kp, vp = cc.layout_from_kv_tensors(dense)
    assert (lay.block_stride, lay.head_bytes) == (0, 0)           # the reference layout
    assert vp == [p + nb * bs * unit for p in kp]
    # FlashAttention with HND blocks: a permuted view of [2, nb, heads, bs, dim]
    H, hb = unit // head_bytes_of(case), head_bytes_of(case)
    phys = torch.zeros(2 * nb * H * bs * hb // 2, dtype=torch.int16)
    view = phys.view(2, nb, H, bs, hb // 2).permute(0, 1, 3, 2, 4)
    lay, _, _ = cc.layout_from_kv_tensors([view])
    assert (lay.block_stride, lay.head_bytes) == (bs * unit, hb)


def test_mla_latent_and_rejected_forms():
    t = torch.zeros(8, 64, 576, dtype=torch.int16)
    lay, kp, vp = cc.layout_from_kv_tensors([t, t.clone()])
    assert (lay.kv, lay.block_stride, lay.head_bytes, vp) == (1, 0, 0, None)
    # a cache of 2 blocks: [2, 2, ...] is ambiguous unless the layout is named
    amb = torch.zeros(2, 2, 16, 8, 128, dtype=torch.int16)
    with pytest.raises(ValueError, match="ambiguous"):
        cc.layout_from_kv_tensors([amb])
    lay, _, vp = cc.layout_from_kv_tensors([amb], kv_layout="flashinfer")
    assert lay.block_stride == 2 * 16 * 2048 and vp[0] == amb.data_ptr() + 16 * 2048
    # dims split across the head / dim axes: not a layout the kernels address
    bad = torch.zeros(2, 4, 16, 128, 8, dtype=torch.int16).transpose(3, 4)
    with pytest.raises(ValueError):
        cc.layout_from_kv_tensors([bad])
    with pytest.raises(ValueError):
        cc.layout_from_kv_tensors([torch.zeros(2, 4, 16, 8, 128), torch.zeros(2, 4, 16, 8, 64)])


# ---- register-time validation ----------------------------------------------

def test_register_paged_rejects_bad_geometry():
    case = next(c for c in CASES if c["name"] == "gqa_bs16")
    unit, bs = gen.unit_of(case), case["block_size"]
    cc.init(case["chunk_size"], 2 * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    try:
        phys, views = fi_tensors(case, True)
        lay, kp, vp = cc.layout_from_kv_tensors(views)
        for stride, hb in [(bs * unit - 16, 0), (2 * bs * unit, 96)]:
            w = cc.Worker("m", lay, kp, vp)
            assert lib.cache_register_paged(C.byref(w.ctx), stride, hb) == -errno.EINVAL
        w = cc.Worker("m", lay, kp, vp)
        w.register()
        assert w.lookup(keys_for(1)) == 0
        w.unregister()
    finally:
        cc.exit()


# ---- record bytes ----------------------------------------------------------

@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_flashinfer_store_writes_the_reference_records(case, hnd, tmp_path, golden_records):
    """records written from a FlashInfer cache are the reference layout's
    golden records byte for byte (read back from the disk tier's files)"""
    root = tmp_path / "kv"
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), str(root), CACHE_BACKEND_MEM)
    try:
        phys, views = fi_tensors(case, hnd)
        lay, kp, vp = cc.layout_from_kv_tensors(views)
        w = cc.Worker("m", lay, kp, vp)
        w.register()
        keys = keys_for(case["chunks"], seed=5)
        assert w.store(keys, gen.block_ids(case)) == 0
        w.flush()
        digests = [hashlib.sha256((root / "m.tp1.0" / k.hex()).read_bytes()).hexdigest() for k in keys]
        assert digests == golden_records[case["name"]]["record_sha256"]
        w.unregister()
    finally:
        cc.exit()


@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_records_cross_between_flash_attn_and_flashinfer(case, hnd):
    """a FlashAttention worker stores, a FlashInfer worker of the same model
    loads at another block table (and back): every byte lands where the
    oracle puts it in the reference layout"""
    cc.init(case["chunk_size"], (2 * case["chunks"] + 1) * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    try:
        unit, bs = gen.unit_of(case), case["block_size"]
        k, v = gen.paged_layers(case)
        fa = [as_flash_attn_view(case, torch.from_numpy(a), torch.from_numpy(b)) for a, b in zip(k, v)]
        wa = cc.Worker("m", *cc.layout_from_kv_tensors(fa))
        wa.register()
        phys, views = fi_tensors(case, hnd, zero=True)
        wf = cc.Worker("m", *cc.layout_from_kv_tensors(views))
        wf.register()
        keys = keys_for(case["chunks"], seed=6)
        bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
        assert wa.store(keys, bids) == 0
        assert wf.load(keys, b2) == 0
        recs = ok.gather(k, v, bids, case["chunk_size"], bs, unit)
        ek, ev = gen.paged_layers(case, zero=True)
        ok.scatter(recs, ek, ev, b2, case["chunk_size"], bs, unit)
        got_k, got_v = from_flashinfer(case, [p.numpy() for p in phys], hnd)
        assert all(np.array_equal(a, b) for a, b in zip(got_k, ek))
        assert all(np.array_equal(a, b) for a, b in zip(got_v, ev))
        # and back: the FlashInfer worker stores, a zeroed FlashAttention cache loads
        keys2 = keys_for(case["chunks"], seed=7)
        assert wf.store(keys2, b2) == 0
        zk, zv = gen.paged_layers(case, zero=True)
        fz = [as_flash_attn_view(case, torch.from_numpy(a), torch.from_numpy(b)) for a, b in zip(zk, zv)]
        wz = cc.Worker("m", *cc.layout_from_kv_tensors(fz))
        wz.register()
        assert wz.load(keys2, bids) == 0
        exp_k, exp_v = gen.paged_layers(case, zero=True)
        ok.scatter(ok.gather(ek, ev, b2, case["chunk_size"], bs, unit), exp_k, exp_v, bids,
                   case["chunk_size"], bs, unit)
        got = [t.view(torch.uint8).reshape(2, -1).numpy() for t in fz]
        assert all(np.array_equal(g[0], e) for g, e in zip(got, exp_k))
        assert all(np.array_equal(g[1], e) for g, e in zip(got, exp_v))
        for w in (wz, wf, wa):
            w.unregister()
    finally:
        cc.exit()


@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
def test_flashinfer_layerwise_async_on_mem_backend(hnd):
    """the layer-ranged API with a head-major cache: layers moved one by one
    in reverse order land as a whole-record load does"""
    case = next(c for c in CASES if c["name"] == "tp8_shard")
    cc.init(case["chunk_size"], (case["chunks"] + 1) * gen.record_bytes(case), None, CACHE_BACKEND_MEM)
    try:
        unit, bs = gen.unit_of(case), case["block_size"]
        phys_s, views_s = fi_tensors(case, hnd)
        ws = cc.Worker("m", *cc.layout_from_kv_tensors(views_s))
        ws.register()
        phys_d, views_d = fi_tensors(case, hnd, zero=True)
        wd = cc.Worker("m", *cc.layout_from_kv_tensors(views_d))
        wd.register()
        keys = keys_for(case["chunks"], seed=8)
        bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
        h = ws.store_async(keys, bids)
        for l in range(case["num_layers"]):
            h.layers(l, l + 1)
        assert h.finish() == 0
        h = wd.load_async(keys, b2)
        for l in reversed(range(case["num_layers"])):
            h.layers(l, l + 1)
        assert h.finish() == 0
        k, v = gen.paged_layers(case)
        ek, ev = gen.paged_layers(case, zero=True)
        ok.scatter(ok.gather(k, v, bids, case["chunk_size"], bs, unit), ek, ev, b2, case["chunk_size"], bs, unit)
        got_k, got_v = from_flashinfer(case, [p.numpy() for p in phys_d], hnd)
        assert all(np.array_equal(a, b) for a, b in zip(got_k, ek))
        assert all(np.array_equal(a, b) for a, b in zip(got_v, ev))
        wd.unregister()
        ws.unregister()
    finally:
        cc.exit()


# ---- wire format -----------------------------------------------------------

def test_register_geometry_trailer_roundtrip():
    keys = [(bytes([i]) * 72, bytes([100 + i]) * 72) for i in range(3)]
    plain = P.encode_register(4, 9, 2, 1, 100, 16, 2, 1024, 72, "llama", keys)
    m = P.decode_request(plain)
    assert (m.block_stride, m.head_bytes) == (0, 0)
    geo = P.encode_register(4, 9, 2, 1, 100, 16, 2, 1024, 72, "llama", keys, 65536, 256)
    assert geo[:12] != plain[:12] and geo[12:len(plain)] == plain[12:]      # only len and the trailer differ
    m = P.decode_request(geo)
    assert (m.block_stride, m.head_bytes) == (65536, 256)
    assert m.k_keys == b"".join(k for k, _ in keys) and m.v_keys == b"".join(v for _, v in keys)
    with pytest.raises(P.ProtocolError):
        P.decode_request(plain + b"junk")
