"""kv_copy_noalloc: the gather/scatter for callers that cannot allocate device
memory (an engine whose paged KV cache and caching allocator already hold all
free HBM, or an embedder whose allocator owns every device byte).  Called
through the C ABI and checked byte for byte against the existing entry point
kv_copy_launch on the same inputs, on two calls in a row.

This file is collected last on purpose: the entry point keeps a static device
array for the life of the process, and a failure here should not stop a
`-x` run before every other test has run.  It must pass alone in a fresh
process and after the other tests."""
import ctypes as C
import errno

import numpy as np
import pytest
import torch

from demo_b200._lib import KVCOPY_ERR_SLOT_RANGE, KvCopyDesc, lib
from tests.golden import gen

pytestmark = pytest.mark.gpu

MAX_LAYERS, MAX_RECORDS, MAX_BLOCKS = 256, 4096, 65536


def _layers(case, seed=None):
    k, v = gen.paged_layers(case, seed=seed)
    kd = [torch.from_numpy(a).cuda() for a in k]
    vd = [torch.from_numpy(a).cuda() for a in v] if v is not None else None
    return kd, vd


def _existing(case, kd, vd, recs, bids, direction):
    """the existing entry point: device arrays + caller-provided error word"""
    kp = torch.tensor([t.data_ptr() for t in kd], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vd], dtype=torch.int64, device="cuda") if vd else None
    rp = torch.tensor([r.data_ptr() for r in recs], dtype=torch.int64, device="cuda")
    bd = torch.from_numpy(bids.astype(np.int64)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = KvCopyDesc(layer_k=kp.data_ptr(), layer_v=vp.data_ptr() if vp is not None else None,
                   records=rp.data_ptr(), slots=None, block_ids=bd.data_ptr(), error=err.data_ptr(),
                   page_buffer_size=case["num_blocks"] * case["block_size"], unit_bytes=gen.unit_of(case),
                   num_tokens=case["chunk_size"], block_size=case["block_size"],
                   num_layers=case["num_layers"], num_records=len(recs), direction=direction)
    assert lib.kv_copy_launch(C.byref(d), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def _noalloc(case, kd, vd, recs, bids, direction, stream=None):
    """the no-allocation entry point: host arrays only"""
    kp = np.array([t.data_ptr() for t in kd], dtype=np.uint64)
    vp = np.array([t.data_ptr() for t in vd], dtype=np.uint64) if vd else None
    rp = np.array([r.data_ptr() for r in recs], dtype=np.uint64)
    b = np.ascontiguousarray(bids.astype(np.uint64))
    s = stream.cuda_stream if stream is not None else None
    return lib.kv_copy_noalloc(torch.cuda.current_device(), kp.ctypes.data,
                               vp.ctypes.data if vp is not None else None, rp.ctypes.data, b.ctypes.data,
                               len(recs), case["num_blocks"] * case["block_size"], gen.unit_of(case),
                               case["chunk_size"], case["block_size"], case["num_layers"], direction, s)


@pytest.mark.parametrize("case", [gen.KV_CASES[1], gen.KV_CASES[2], gen.KV_CASES[4]], ids=lambda c: c["name"])
def test_noalloc_matches_existing_entry_point_two_calls_in_a_row(case):
    kd, vd = _layers(case)
    rb = gen.record_bytes(case)
    n = case["chunks"]
    stream = torch.cuda.Stream()
    # call 1: gather at block table A; call 2: gather at block table B (the
    # scratch array still holds call 1's metadata when call 2 starts)
    for call, off in enumerate((0, 1)):
        bids = gen.block_ids(case, seed_offset=off)
        ref = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(n)]
        got = [torch.full((rb,), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(n)]
        _existing(case, kd, vd, ref, bids, 1)
        assert _noalloc(case, kd, vd, got, bids, 1, stream) == 0, call
        for a, b in zip(ref, got):
            assert torch.equal(a, b), call
    # and the scatter direction, twice
    for call in range(2):
        recs = [torch.from_numpy(r).cuda() for r in gen.records_for_scatter(case)]
        bids = gen.block_ids(case, seed_offset=2 + call)
        k1, v1 = _layers(case, seed=7)
        k2, v2 = _layers(case, seed=7)
        _existing(case, k1, v1, recs, bids, 0)
        assert _noalloc(case, k2, v2, recs, bids, 0) == 0
        assert all(torch.equal(a, b) for a, b in zip(k1, k2))
        if v1 is not None:
            assert all(torch.equal(a, b) for a, b in zip(v1, v2))


def test_noalloc_errors_and_limits():
    case = gen.KV_CASES[1]
    kd, vd = _layers(case)
    rb = gen.record_bytes(case)
    recs = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    bad = gen.block_ids(case).copy()
    bad[5] = case["num_blocks"] + 3                    # past the end of the paged cache
    assert _noalloc(case, kd, vd, recs, bad, 1) == -errno.EINVAL
    # the error word is cleared per call: a good call right after succeeds
    good = gen.block_ids(case)
    ref = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    _existing(case, kd, vd, ref, good, 1)
    assert _noalloc(case, kd, vd, recs, good, 1) == 0
    assert all(torch.equal(a, b) for a, b in zip(ref, recs))
    # sizes beyond the static scratch are rejected before touching the GPU
    big = dict(case, chunks=MAX_RECORDS + 1)
    fake = [recs[0]] * (MAX_RECORDS + 1)
    assert _noalloc(big, kd, vd, fake, np.zeros((MAX_RECORDS + 1) * 16, np.uint64), 1) == -errno.E2BIG
    many_layers = dict(case, num_layers=MAX_LAYERS + 1)
    assert _noalloc(many_layers, kd * 100, vd * 100, recs, good, 1) == -errno.E2BIG
    assert lib.kv_copy_noalloc(0, None, None, None, None, 1, 1, 1, 1, 1, 1, 1, None) == -errno.EINVAL
