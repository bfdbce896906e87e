"""A seeded sweep of record geometries through kv_copy_launch on both kernel
paths, gather and scatter, against the oracle (the C restatement of
CrossCache's mem.cpp record layout): units from 6 bytes to 4 KiB, blocks of
1 to 64 tokens, records of 1 to 32 blocks, K+V and K-only caches.  Among
them are TMA bulk shapes whose tiles do not divide a record's blocks (a
10 KiB block run: 3 blocks a 32 KiB tile, then a 1-block tail tile), which
the five golden shapes never reach."""
import ctypes as C

import numpy as np
import pytest
import torch

from demo_b200._lib import KVCOPY_FLAG_BULK, KVCOPY_PATH_BULK, KVCOPY_PATH_REGISTER, KvCopyDesc, lib
from oracle import kvcopy as ok
from tests.golden import gen
from tests.gpu_util import ptr_array, to_dev

pytestmark = pytest.mark.gpu

UNITS = [6, 16, 48, 256, 640, 768, 1024, 1152, 2048, 4096]
BLOCK_SIZES = [1, 2, 4, 8, 16, 32, 64]
# bulk shapes that the golden cases do not reach: (unit, block size, tokens
# per record), block runs of 8-32 KiB, most leaving a partial last tile
FORCED = [(640, 16, 256), (768, 16, 80), (1152, 8, 256), (2560, 4, 64), (2048, 8, 64)]


def _case(seed: int) -> dict:
    rng = np.random.default_rng(9000 + seed)
    if seed < len(FORCED):
        unit, bs, chunk = FORCED[seed]
    else:
        unit, bs = int(rng.choice(UNITS)), int(rng.choice(BLOCK_SIZES))
        chunk = bs * int(rng.choice([1, 2, 4, 8, 16]))
        while chunk * unit * 4 > (8 << 20):          # keep one record's layer part small
            chunk //= 2
        chunk = max(chunk, bs)
    records = int(rng.integers(1, 6))
    used = records * (chunk // bs)
    return dict(name=f"r{seed}", num_blocks=2 * used + int(rng.integers(0, 8)), block_size=bs, chunk_size=chunk,
                num_layers=int(rng.integers(1, 5)), hidden=unit // 2 if unit % 2 == 0 else unit, elt=2 if unit % 2 == 0 else 1,
                kv=int(rng.choice([1, 2])), chunks=records, seed=300 + seed)


def _launch(case, k, v, recs, bids, direction, flags):
    kp = ptr_array(k)
    vp = ptr_array(v) if v is not None else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    bd = to_dev(bids.astype(np.int64))
    d = KvCopyDesc(layer_k=kp.data_ptr(), layer_v=vp.data_ptr() if vp is not None else None,
                   records=ptr_array(recs).data_ptr(), slots=None, block_ids=bd.data_ptr(), error=err.data_ptr(),
                   page_buffer_size=case["num_blocks"] * case["block_size"], unit_bytes=gen.unit_of(case),
                   num_tokens=case["chunk_size"], block_size=case["block_size"], num_layers=case["num_layers"],
                   num_records=len(recs), direction=direction, flags=flags)
    path = lib.kv_copy_path(C.byref(d))
    assert lib.kv_copy_launch(C.byref(d), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return path


@pytest.mark.parametrize("flags", [0, KVCOPY_FLAG_BULK], ids=["register", "bulk"])
@pytest.mark.parametrize("seed", range(24))
def test_random_geometry_gather_and_scatter_match_oracle(seed, flags):
    case = _case(seed)
    unit, bs = gen.unit_of(case), case["block_size"]
    k, v = gen.paged_layers(case)
    kd = [to_dev(a) for a in k]
    vd = [to_dev(a) for a in v] if v is not None else None
    bids = gen.block_ids(case)
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    path = _launch(case, kd, vd, recs, bids, 1, flags)
    run = bs * unit
    bulk_shape = unit % 16 == 0 and 8192 <= run <= 32768
    assert path == (KVCOPY_PATH_BULK if flags and bulk_shape else KVCOPY_PATH_REGISTER), (case, path)
    exp = ok.gather(k, v, bids, case["chunk_size"], bs, unit)
    for r, e in zip(recs, exp):
        assert np.array_equal(r.cpu().numpy(), e), case
    # scatter the records into empty layers at another block table
    zk, zv = gen.paged_layers(case, zero=True)
    zkd = [to_dev(a) for a in zk]
    zvd = [to_dev(a) for a in zv] if zv is not None else None
    bids2 = gen.block_ids(case, seed_offset=1)
    _launch(case, zkd, zvd, recs, bids2, 0, flags)
    ok.scatter(exp, zk, zv, bids2, case["chunk_size"], bs, unit)
    assert all(np.array_equal(t.cpu().numpy(), e) for t, e in zip(zkd, zk)), case
    if zv is not None:
        assert all(np.array_equal(t.cpu().numpy(), e) for t, e in zip(zvd, zv)), case


def test_the_sweep_reaches_partial_bulk_tiles():
    """at least the forced shapes take the bulk path with a tail tile"""
    tails = 0
    for seed in range(24):
        c = _case(seed)
        run = c["block_size"] * gen.unit_of(c)
        if gen.unit_of(c) % 16 == 0 and 8192 <= run <= 32768:
            gpt = 32768 // run
            bpr = c["chunk_size"] // c["block_size"]
            tails += (bpr % gpt) != 0
    assert tails >= 4
