"""Parity of the sm_100a gather/scatter kernel and the CUDA adaptor ABI with
the oracle and with the golden digests of CrossCache's own mem.cpp."""
import ctypes as C
import errno
import os

import numpy as np
import pytest
import torch

from demo_b200._lib import (KVCOPY_ERR_SLOT_RANGE, KVCOPY_FLAG_BULK, KvCopyDesc, TransferBatch,
                            TransferParams, lib)
from oracle import kvcopy as ok
from tests.golden import gen
from tests.gpu_util import DeviceKV, dsha, ptr_array, to_dev

pytestmark = pytest.mark.gpu


def launch(kv: DeviceKV, records, bids=None, slots=None, direction=1, err=None, num_records=None, flags=0):
    case = kv.case
    recp = ptr_array(records)
    d = KvCopyDesc(layer_k=kv.kp.data_ptr(), layer_v=kv.vp.data_ptr() if kv.vp is not None else None,
                   records=recp.data_ptr(),
                   slots=slots.data_ptr() if slots is not None else None,
                   block_ids=bids.data_ptr() if bids is not None else None,
                   error=err.data_ptr() if err is not None else None,
                   page_buffer_size=case["num_blocks"] * case["block_size"],
                   unit_bytes=gen.unit_of(case), num_tokens=case["chunk_size"],
                   block_size=case["block_size"], num_layers=case["num_layers"],
                   num_records=len(records) if num_records is None else num_records,
                   direction=direction, flags=flags)
    ret = lib.kv_copy_launch(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return ret


@pytest.mark.parametrize("flags", [0, KVCOPY_FLAG_BULK], ids=["lsu", "bulk"])
@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_gather_block_mode_matches_reference_golden(case, flags, golden_records):
    kv = DeviceKV(case)
    bids = gen.block_ids(case)
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert launch(kv, recs, bids=to_dev(bids.astype(np.int64)), err=err, flags=flags) == 0
    assert int(err.item()) == 0
    assert [dsha(r) for r in recs] == golden_records[case["name"]]["record_sha256"]


@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_gather_slot_mode_matches_oracle(case):
    kv = DeviceKV(case)
    bids = gen.block_ids(case)
    slots = ok.slot_mapping(bids, case["block_size"])
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    assert launch(kv, recs, slots=to_dev(slots)) == 0
    k, v = gen.paged_layers(case)
    exp = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    for r, e in zip(recs, exp):
        assert np.array_equal(r.cpu().numpy(), e)


@pytest.mark.parametrize("flags", [0, KVCOPY_FLAG_BULK], ids=["lsu", "bulk"])
@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_scatter_matches_reference_golden(case, flags, golden_records):
    kv = DeviceKV(case, zero=True)
    bids2 = gen.block_ids(case, seed_offset=1)
    recs = [to_dev(r) for r in gen.records_for_scatter(case)]
    assert launch(kv, recs, bids=to_dev(bids2.astype(np.int64)), direction=0, flags=flags) == 0
    g = golden_records[case["name"]]
    assert [dsha(t) for t in kv.k] == g["scatter_k_sha256"]
    if kv.v is not None:
        assert [dsha(t) for t in kv.v] == g["scatter_v_sha256"]


def test_random_slots_and_unaligned_bases_match_oracle():
    """arbitrary per-token slots, odd units, and record/layer bases that are
    not 16-byte aligned (byte-wise tile path)"""
    rng = np.random.default_rng(8)
    for trial in range(6):
        L = int(rng.integers(1, 4))
        hidden, elt = int(rng.integers(1, 300)), int(rng.choice([1, 2, 4]))
        unit = hidden * elt
        C_, nslots = int(rng.integers(1, 40)), 200
        case = dict(num_blocks=nslots, block_size=1, chunk_size=C_, num_layers=L, hidden=hidden,
                    elt=elt, kv=2, chunks=2, seed=100 + trial)
        k, v = gen.paged_layers(case)
        off = int(rng.integers(0, 3)) if trial % 2 else 0
        kd = [to_dev(np.concatenate([np.zeros(off, np.uint8), a]))[off:] for a in k]
        vd = [to_dev(np.concatenate([np.zeros(off, np.uint8), a]))[off:] for a in v]
        kv = DeviceKV.__new__(DeviceKV)
        kv.case, kv.k, kv.v, kv.kp, kv.vp = case, kd, vd, ptr_array(kd), ptr_array(vd)
        slots = rng.integers(0, nslots, 2 * C_).astype(np.int64)
        rb = 2 * L * C_ * unit
        big = torch.zeros(2 * rb + 8, dtype=torch.uint8, device="cuda")
        recs = [big[off: off + rb], big[rb + 2 * off: 2 * rb + 2 * off]]
        assert launch(kv, recs, slots=to_dev(slots)) == 0
        for i in range(2):
            e = np.zeros(rb, np.uint8)
            ok.transfer(e, k, v, slots[i * C_:(i + 1) * C_], C_, hidden, elt, True)
            assert np.array_equal(recs[i].cpu().numpy(), e), (trial, i)


@pytest.mark.parametrize("flags", [0, KVCOPY_FLAG_BULK], ids=["lsu", "bulk"])
def test_out_of_range_block_sets_error_and_copies_the_rest(flags):
    case = gen.KV_CASES[1]
    kv = DeviceKV(case)
    bids = gen.block_ids(case).astype(np.int64)
    bad = bids.copy()
    bad[3] = case["num_blocks"]              # one block id past the end
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert launch(kv, recs, bids=to_dev(bad), err=err, flags=flags) == 0
    assert int(err.item()) & KVCOPY_ERR_SLOT_RANGE
    k, v = gen.paged_layers(case)
    exp = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    for i in (1, 2):          # chunks without the bad block are exact
        assert np.array_equal(recs[i].cpu().numpy(), exp[i])


def test_invalid_descriptors_rejected():
    case = gen.KV_CASES[0]
    kv = DeviceKV(case)
    rec = torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda")
    bids = to_dev(gen.block_ids(case).astype(np.int64))
    d = KvCopyDesc(layer_k=kv.kp.data_ptr(), layer_v=None, records=ptr_array([rec]).data_ptr(),
                   slots=None, block_ids=None, error=None, page_buffer_size=80, unit_bytes=8192,
                   num_tokens=4, block_size=2, num_layers=2, num_records=1, direction=1)
    assert lib.kv_copy_launch(C.byref(d), None) == -errno.EINVAL        # neither slots nor block ids
    d.block_ids = bids.data_ptr()
    d.num_tokens = 5                                                      # not a block multiple
    assert lib.kv_copy_launch(C.byref(d), None) == -errno.EINVAL
    d.num_tokens = 4
    d.num_records = 0
    assert lib.kv_copy_launch(C.byref(d), None) == 0                      # empty batch
    assert lib.kv_copy_payload_bytes(C.byref(d)) == 0


# ---------------------------------------------------------------------------
# adaptor ABI (include/device.h)

@pytest.fixture
def cuda_adaptor():
    ad = lib.cuda_adaptor_create()
    assert ad
    yield ad
    lib.cuda_adaptor_destroy(ad)


def open_layers(ad, kv: DeviceKV):
    kp = np.array([t.data_ptr() for t in kv.k], np.uint64)
    dk = lib.open_ipc_keys(ad, 0, 8, len(kp), kp.ctypes.data)
    dv = None
    if kv.v is not None:
        vp = np.array([t.data_ptr() for t in kv.v], np.uint64)
        dv = lib.open_ipc_keys(ad, 0, 8, len(vp), vp.ctypes.data)
    assert dk and (kv.v is None or dv)
    return dk, dv


@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
@pytest.mark.parametrize("where", ["pinned_host", "device"])
def test_transfer_kvcache_per_chunk_abi(case, where, cuda_adaptor, golden_records):
    """reference call shape: one record per call, slot mapping uploaded with
    wrapper_ptr, record in the pinned pool (device alias) or in HBM"""
    ad = cuda_adaptor
    src, dst = DeviceKV(case), DeviceKV(case, zero=True)
    sk, sv = open_layers(ad, src)
    dk, dv = open_layers(ad, dst)
    bids = gen.block_ids(case)
    bpc = case["chunk_size"] // case["block_size"]
    rb = gen.record_bytes(case)
    if where == "pinned_host":
        size = (rb + 4095) // 4096 * 4096
        daddr = C.c_void_p()
        host = lib.alloc_pinned_ptr(ad, 0, size, 0, C.byref(daddr))
        assert host
        rec_np = np.ctypeslib.as_array((C.c_uint8 * rb).from_address(host))
        caches, caches_h = daddr.value, host
    else:
        rec_t = torch.zeros(rb, dtype=torch.uint8, device="cuda")
        caches = caches_h = rec_t.data_ptr()
    exp_k, exp_v = gen.paged_layers(case, zero=True)
    for c in range(case["chunks"]):
        cb = bids[c * bpc:(c + 1) * bpc]
        slots = ok.slot_mapping(cb, case["block_size"])
        ds = lib.wrapper_ptr(ad, 0, slots.ctypes.data, slots.nbytes)
        assert ds
        p = TransferParams(caches=caches, caches_h=caches_h, keys_ptrs=sk, value_ptrs=sv,
                           page_buffer_size=case["num_blocks"] * case["block_size"], slot_mapping=ds,
                           devid=0, caches_element_size=case["elt"], num_layers=case["num_layers"],
                           num_tokens=case["chunk_size"], hidden_dim_size=case["hidden"], direction=True)
        assert lib.transfer_kvcache(ad, C.byref(p)) == 0
        got = rec_np.copy() if where == "pinned_host" else rec_t.cpu().numpy()
        assert gen.sha(got) == golden_records[case["name"]]["record_sha256"][c]
        p.keys_ptrs, p.value_ptrs, p.direction = dk, dv, False
        assert lib.transfer_kvcache(ad, C.byref(p)) == 0
        ok.scatter([got], exp_k, exp_v, cb, case["chunk_size"], case["block_size"], gen.unit_of(case))
        lib.unwrapper_ptr(ad, ds)
    kh, vh = dst.host()
    assert all(np.array_equal(a, b) for a, b in zip(kh, exp_k))
    if vh is not None:
        assert all(np.array_equal(a, b) for a, b in zip(vh, exp_v))
    if where == "pinned_host":
        lib.free_pinned_ptr(ad, host, size)
    for h in (sk, sv, dk, dv):
        if h:
            lib.close_ipc_keys(ad, h)


def run_batch(ad, kv, recs_ptrs, bids, direction, on_device=False):
    case = kv.case
    dk, dv = open_layers(ad, kv)
    arr = (C.c_void_p * len(recs_ptrs))(*recs_ptrs)
    b = np.ascontiguousarray(bids.astype(np.uint64))
    tb = TransferBatch(keys_ptrs=dk, value_ptrs=dv,
                       page_buffer_size=case["num_blocks"] * case["block_size"],
                       records=arr, block_ids=b.ctypes.data_as(C.POINTER(C.c_uint64)),
                       num_records=len(recs_ptrs), block_size=case["block_size"],
                       hidden_dim_size=case["hidden"], num_layers=case["num_layers"],
                       num_tokens=case["chunk_size"], devid=0, caches_element_size=case["elt"],
                       record_on_device=1 if on_device else 0, direction=direction)
    ret = lib.transfer_kvcache_batch(ad, C.byref(tb))
    lib.close_ipc_keys(ad, dk)
    if dv:
        lib.close_ipc_keys(ad, dv)
    return ret


@pytest.mark.parametrize("mode", ["staged", "direct", "device"])
@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_transfer_batch_roundtrip(case, mode, golden_records, monkeypatch):
    if mode == "direct":
        monkeypatch.setenv("CROSSCACHE_XFER_MODE", "direct")
    ad = lib.cuda_adaptor_create()
    try:
        kv = DeviceKV(case)
        rb = gen.record_bytes(case)
        n = case["chunks"]
        if mode == "device":
            store = torch.zeros(n * rb, dtype=torch.uint8, device="cuda")
            ptrs = [store.data_ptr() + i * rb for i in range(n)]
        else:
            size = (n * rb + 4095) // 4096 * 4096
            daddr = C.c_void_p()
            host = lib.alloc_pinned_ptr(ad, 0, size, 0, C.byref(daddr))
            assert host
            hv = np.ctypeslib.as_array((C.c_uint8 * (n * rb)).from_address(host))
            hv[:] = 0xAB
            ptrs = [host + i * rb for i in range(n)]
        bids = gen.block_ids(case)
        assert run_batch(ad, kv, ptrs, bids, True, mode == "device") == 0
        flat = store.cpu().numpy() if mode == "device" else hv.copy()
        got = [gen.sha(flat[i * rb:(i + 1) * rb]) for i in range(n)]
        assert got == golden_records[case["name"]]["record_sha256"]
        # load the golden scatter records into zeroed layers
        dst = DeviceKV(case, zero=True)
        for i, r in enumerate(gen.records_for_scatter(case)):
            if mode == "device":
                store[i * rb:(i + 1) * rb].copy_(torch.from_numpy(r))
            else:
                hv[i * rb:(i + 1) * rb] = r
        assert run_batch(ad, dst, ptrs, gen.block_ids(case, seed_offset=1), False, mode == "device") == 0
        g = golden_records[case["name"]]
        assert [dsha(t) for t in dst.k] == g["scatter_k_sha256"]
        if dst.v is not None:
            assert [dsha(t) for t in dst.v] == g["scatter_v_sha256"]
        # a bad block id fails the whole call with -EINVAL
        bad = bids.copy()
        bad[0] = case["num_blocks"] + 5
        assert run_batch(ad, kv, ptrs, bad, True, mode == "device") == -errno.EINVAL
        if mode != "device":
            lib.free_pinned_ptr(ad, host, size)
    finally:
        lib.cuda_adaptor_destroy(ad)


def test_staging_ring_many_records_larger_than_ring(cuda_adaptor):
    """more record groups than the staging ring has sub-slots (wrap-around)"""
    case = dict(num_blocks=2048, block_size=16, chunk_size=256, num_layers=8, hidden=1024, elt=2,
                kv=2, chunks=40, seed=31)
    kv = DeviceKV(case)
    rb = gen.record_bytes(case)      # 8 MiB records, 4 per 32 MiB sub-slot
    n = case["chunks"]
    size = n * rb
    daddr = C.c_void_p()
    host = lib.alloc_pinned_ptr(cuda_adaptor, 0, size, 0, C.byref(daddr))
    hv = np.ctypeslib.as_array((C.c_uint8 * size).from_address(host))
    bids = gen.block_ids(case)
    ptrs = [host + i * rb for i in range(n)]
    assert run_batch(cuda_adaptor, kv, ptrs, bids, True) == 0
    k, v = gen.paged_layers(case)
    exp = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case), nthreads=8)
    for i in range(n):
        assert np.array_equal(hv[i * rb:(i + 1) * rb], exp[i]), i
    dst = DeviceKV(case, zero=True)
    bids2 = gen.block_ids(case, seed_offset=1)
    assert run_batch(cuda_adaptor, dst, ptrs, bids2, False) == 0
    ek, ev = gen.paged_layers(case, zero=True)
    ok.scatter(exp, ek, ev, bids2, case["chunk_size"], case["block_size"], gen.unit_of(case), nthreads=8)
    kh, vh = dst.host()
    assert all(np.array_equal(a, b) for a, b in zip(kh, ek))
    assert all(np.array_equal(a, b) for a, b in zip(vh, ev))
    lib.free_pinned_ptr(cuda_adaptor, host, size)


def test_bulk_scatter_skips_bad_block_and_writes_the_rest():
    # 1 KiB units x 16 tokens = 16 KiB runs: 2 blocks per 32 KiB bulk tile
    case = dict(num_blocks=128, block_size=16, chunk_size=256, num_layers=3, hidden=512, elt=2,
                kv=2, chunks=4, seed=16)
    kv = DeviceKV(case, zero=True)
    bids = gen.block_ids(case).astype(np.int64)
    bad = bids.copy()
    bad[5] = case["num_blocks"] + 1
    recs = [to_dev(r) for r in gen.records_for_scatter(case)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert launch(kv, recs, bids=to_dev(bad), err=err, direction=0, flags=KVCOPY_FLAG_BULK) == 0
    assert int(err.item()) & KVCOPY_ERR_SLOT_RANGE
    # every other block holds exactly what the oracle writes with the good table;
    # the block the bad id replaced is never written
    ek, ev = gen.paged_layers(case, zero=True)
    ok.scatter(gen.records_for_scatter(case), ek, ev, bids.astype(np.uint64), case["chunk_size"],
               case["block_size"], gen.unit_of(case))
    kh, vh = kv.host()
    blk = case["block_size"] * gen.unit_of(case)
    keep = [int(b) for i, b in enumerate(bids) if i != 5]
    for a, e in zip(kh + vh, ek + ev):
        assert np.array_equal(a.reshape(-1, blk)[keep], e.reshape(-1, blk)[keep])
        assert not a.reshape(-1, blk)[int(bids[5])].any()


def test_bulk_path_matches_lsu_on_large_random_tables():
    """many tiles per CTA (pipeline wrap-around of the 4-stage ring)"""
    case = dict(num_blocks=4096, block_size=16, chunk_size=256, num_layers=8, hidden=1024, elt=2,
                kv=2, chunks=96, seed=77)
    kv = DeviceKV(case)
    bids = to_dev(gen.block_ids(case).astype(np.int64))
    rb = gen.record_bytes(case)
    a = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    b = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    assert launch(kv, a, bids=bids) == 0
    assert launch(kv, b, bids=bids, flags=KVCOPY_FLAG_BULK) == 0
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    dst1, dst2 = DeviceKV(case, zero=True), DeviceKV(case, zero=True)
    bids2 = to_dev(gen.block_ids(case, seed_offset=1).astype(np.int64))
    assert launch(dst1, a, bids=bids2, direction=0) == 0
    assert launch(dst2, a, bids=bids2, direction=0, flags=KVCOPY_FLAG_BULK) == 0
    assert all(torch.equal(x, y) for x, y in zip(dst1.k + dst1.v, dst2.k + dst2.v))


def test_kernel_launch_counter_advances(cuda_adaptor):
    before = lib.crosscache_kernel_launches()
    case = gen.KV_CASES[0]
    kv = DeviceKV(case)
    rec = torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda")
    assert launch(kv, [rec], bids=to_dev(gen.block_ids(case).astype(np.int64))) == 0
    assert lib.crosscache_kernel_launches() == before + 1
