"""kv_copy_noalloc: the gather/scatter for callers that cannot allocate device
memory -- a serving engine whose paged KV cache and caching allocator already
hold all free HBM, or an embedder whose allocator owns every device byte.

Called through the C ABI.  Its records and scattered layers are compared with
the golden digests of CrossCache's own mem.cpp (the same pins the other
kernel tests use) and with the existing entry point kv_copy_launch on the same
inputs, on two calls in a row, on the register path and on the TMA bulk path.
A fresh child process checks the property the entry point exists for: after
its set-up call, gathers and scatters take no page of device memory, and
still succeed once almost all free HBM has been taken.

This file is collected last on purpose: the entry point keeps a static device
array for the life of the process, and a failure here should not stop a
`-x` run before every other test has run.  It passes alone in a fresh process
and after the other tests."""
import ctypes as C
import errno
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from demo_b200._lib import KVCOPY_FLAG_BULK, KVCOPY_FLAG_TEST_STALL, KVCOPY_PATH_BULK, KVCOPY_PATH_REGISTER, \
    KvCopyDesc, lib
from oracle import kvcopy as ok
from tests.golden import gen
from tests.gpu_util import dsha

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
MAX_LAYERS, MAX_RECORDS, MAX_BLOCKS = 256, 4096, 65536
FLAGS = [0, KVCOPY_FLAG_BULK]
FLAG_IDS = ["register", "bulk"]


def _layers(case, seed=None, zero=False):
    k, v = gen.paged_layers(case, seed=seed, zero=zero)
    kd = [torch.from_numpy(a).cuda() for a in k]
    vd = [torch.from_numpy(a).cuda() for a in v] if v is not None else None
    return kd, vd


def _desc(case, kp, vp, rp, bd, err, n, direction, flags):
    return KvCopyDesc(layer_k=kp.data_ptr(), layer_v=vp.data_ptr() if vp is not None else None,
                      records=rp.data_ptr(), slots=None, block_ids=bd.data_ptr(), error=err.data_ptr(),
                      page_buffer_size=case["num_blocks"] * case["block_size"], unit_bytes=gen.unit_of(case),
                      num_tokens=case["chunk_size"], block_size=case["block_size"],
                      num_layers=case["num_layers"], num_records=n, direction=direction, flags=flags)


def _existing(case, kd, vd, recs, bids, direction, flags=0):
    """the existing entry point: device arrays + caller-provided error word"""
    kp = torch.tensor([t.data_ptr() for t in kd], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vd], dtype=torch.int64, device="cuda") if vd else None
    rp = torch.tensor([r.data_ptr() for r in recs], dtype=torch.int64, device="cuda")
    bd = torch.from_numpy(bids.astype(np.int64)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.kv_copy_launch(C.byref(_desc(case, kp, vp, rp, bd, err, len(recs), direction, flags)), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def _path(case, flags):
    """the kernel kv_copy_launch (and so the no-allocation entry point) runs for a case"""
    one = torch.zeros(1, dtype=torch.int64, device="cuda")
    return lib.kv_copy_path(C.byref(_desc(case, one, one if case["kv"] == 2 else None, one, one, one, 1, 1, flags)))


def _noalloc(case, kd, vd, recs, bids, direction, flags=0, stream=None):
    """the no-allocation entry point: host arrays only"""
    kp = np.array([t.data_ptr() for t in kd], dtype=np.uint64)
    vp = np.array([t.data_ptr() for t in vd], dtype=np.uint64) if vd else None
    rp = np.array([r.data_ptr() for r in recs], dtype=np.uint64)
    b = np.ascontiguousarray(bids.astype(np.uint64))
    s = stream.cuda_stream if stream is not None else None
    return lib.kv_copy_noalloc(torch.cuda.current_device(), kp.ctypes.data,
                               vp.ctypes.data if vp is not None else None, rp.ctypes.data, b.ctypes.data,
                               len(recs), case["num_blocks"] * case["block_size"], gen.unit_of(case),
                               case["chunk_size"], case["block_size"], case["num_layers"], direction, flags, s)


@pytest.mark.parametrize("flags", FLAGS, ids=FLAG_IDS)
@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_noalloc_gather_matches_golden_and_existing_entry_point_two_calls(case, flags, golden_records):
    kd, vd = _layers(case)
    rb, n = gen.record_bytes(case), case["chunks"]
    stream = torch.cuda.Stream()
    # call 1: the golden block table, against the mem.cpp record digests
    bids = gen.block_ids(case)
    got = [torch.full((rb,), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(n)]
    assert _noalloc(case, kd, vd, got, bids, 1, flags, stream) == 0
    assert [dsha(r) for r in got] == golden_records[case["name"]]["record_sha256"]
    # call 2, right after (the scratch array still holds call 1's metadata):
    # another block table, against the existing entry point and the oracle
    bids = gen.block_ids(case, seed_offset=5)
    ref = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(n)]
    got = [torch.full((rb,), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(n)]
    _existing(case, kd, vd, ref, bids, 1, flags)
    assert _noalloc(case, kd, vd, got, bids, 1, flags, stream) == 0
    k, v = gen.paged_layers(case)
    exp = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    for a, b, e in zip(ref, got, exp):
        assert torch.equal(a, b)
        assert np.array_equal(b.cpu().numpy(), e)


@pytest.mark.parametrize("flags", FLAGS, ids=FLAG_IDS)
@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_noalloc_scatter_matches_golden_and_existing_entry_point_two_calls(case, flags, golden_records):
    g = golden_records[case["name"]]
    recs = [torch.from_numpy(r).cuda() for r in gen.records_for_scatter(case)]
    bids = gen.block_ids(case, seed_offset=1)          # the golden scatter table
    for call in range(2):
        k1, v1 = _layers(case, zero=True)
        k2, v2 = _layers(case, zero=True)
        _existing(case, k1, v1, recs, bids, 0, flags)
        assert _noalloc(case, k2, v2, recs, bids, 0, flags) == 0, call
        assert [dsha(t) for t in k2] == g["scatter_k_sha256"], call
        assert all(torch.equal(a, b) for a, b in zip(k1, k2)), call
        if v2 is not None:
            assert [dsha(t) for t in v2] == g["scatter_v_sha256"], call
            assert all(torch.equal(a, b) for a, b in zip(v1, v2)), call


def test_noalloc_takes_the_bulk_path_where_the_shapes_allow():
    """the flag reaches the kernel selection: 32 KiB and 16 KiB block runs take
    the TMA bulk kernel, 4 KiB runs and odd units the register kernel"""
    by_name = {c["name"]: c for c in gen.KV_CASES}
    assert _path(by_name["gqa_bs16"], KVCOPY_FLAG_BULK) == KVCOPY_PATH_BULK
    assert _path(by_name["test_copy_defaults"], KVCOPY_FLAG_BULK) == KVCOPY_PATH_BULK
    assert _path(by_name["tp8_shard"], KVCOPY_FLAG_BULK) == KVCOPY_PATH_REGISTER
    assert _path(by_name["odd_unit"], KVCOPY_FLAG_BULK) == KVCOPY_PATH_REGISTER
    assert _path(by_name["gqa_bs16"], 0) == KVCOPY_PATH_REGISTER


def test_noalloc_errors_and_limits(golden_records):
    case = gen.KV_CASES[1]
    kd, vd = _layers(case)
    rb = gen.record_bytes(case)
    recs = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    bad = gen.block_ids(case).copy()
    bad[5] = case["num_blocks"] + 3                    # past the end of the paged cache
    for flags in FLAGS:
        assert _noalloc(case, kd, vd, recs, bad, 1, flags) == -errno.EINVAL
    # the error word is cleared per call: a good call right after succeeds
    good = gen.block_ids(case)
    assert _noalloc(case, kd, vd, recs, good, 1) == 0
    assert [dsha(r) for r in recs] == golden_records[case["name"]]["record_sha256"]
    # sizes beyond the static scratch are rejected before touching the GPU
    big = dict(case, chunks=MAX_RECORDS + 1)
    fake = [recs[0]] * (MAX_RECORDS + 1)
    assert _noalloc(big, kd, vd, fake, np.zeros((MAX_RECORDS + 1) * 16, np.uint64), 1) == -errno.E2BIG
    many_layers = dict(case, num_layers=MAX_LAYERS + 1)
    assert _noalloc(many_layers, kd * 100, vd * 100, recs, good, 1) == -errno.E2BIG
    assert lib.kv_copy_noalloc(0, None, None, None, None, 1, 1, 1, 1, 1, 1, 1, 0, None) == -errno.EINVAL
    # only KVCOPY_FLAG_BULK is accepted (the fault-detection test flag is not)
    assert _noalloc(case, kd, vd, recs, good, 1, KVCOPY_FLAG_BULK | KVCOPY_FLAG_TEST_STALL) == -errno.EINVAL
    # a set-up call: no records, no arrays
    assert lib.kv_copy_noalloc(torch.cuda.current_device(), None, None, None, None, 0, 0, 0, 0, 0, 0, 0, 0,
                               None) == 0
    assert lib.kv_copy_noalloc(64, None, None, None, None, 0, 0, 0, 0, 0, 0, 0, 0, None) == -errno.EINVAL


# The child process: nothing on the device but what it allocates itself.
CHILD = r"""
import json, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from demo_b200._lib import KVCOPY_FLAG_BULK, lib
from tests.golden import gen
from tests.gpu_util import dsha

golden = {c["case"]: c for c in json.loads(open(sys.argv[2]).read())}
dev = torch.cuda.current_device()
cases = [c for c in gen.KV_CASES if c["name"] in ("gqa_bs16", "tp8_shard")]
bufs = []
for case in cases:
    k, v = gen.paged_layers(case)
    kd = [torch.from_numpy(a).cuda() for a in k]
    vd = [torch.from_numpy(a).cuda() for a in v]
    zk = [torch.zeros_like(t) for t in kd]
    zv = [torch.zeros_like(t) for t in vd]
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    srec = [torch.from_numpy(r).cuda() for r in gen.records_for_scatter(case)]
    bufs.append((case, kd, vd, zk, zv, recs, srec))
torch.cuda.synchronize()

def call(case, kd, vd, recs, bids, direction, flags):
    kp = np.array([t.data_ptr() for t in kd], np.uint64)
    vp = np.array([t.data_ptr() for t in vd], np.uint64)
    rp = np.array([r.data_ptr() for r in recs], np.uint64)
    b = np.ascontiguousarray(bids.astype(np.uint64))
    return lib.kv_copy_noalloc(dev, kp.ctypes.data, vp.ctypes.data, rp.ctypes.data, b.ctypes.data, len(recs),
                               case["num_blocks"] * case["block_size"], gen.unit_of(case), case["chunk_size"],
                               case["block_size"], case["num_layers"], direction, flags, None)

def round_trip():
    ok = True
    for case, kd, vd, zk, zv, recs, srec in bufs:
        g = golden[case["name"]]
        for flags in (0, KVCOPY_FLAG_BULK):
            for t in recs + zk + zv:
                t.zero_()
            torch.cuda.synchronize()
            ok &= call(case, kd, vd, recs, gen.block_ids(case), 1, flags) == 0
            ok &= [dsha(r) for r in recs] == g["record_sha256"]
            ok &= call(case, zk, zv, srec, gen.block_ids(case, seed_offset=1), 0, flags) == 0
            ok &= [dsha(t) for t in zk] == g["scatter_k_sha256"] and [dsha(t) for t in zv] == g["scatter_v_sha256"]
    return bool(ok)

free_start = torch.cuda.mem_get_info()[0]
setup = lib.kv_copy_noalloc(dev, None, None, None, None, 0, 0, 0, 0, 0, 0, 0, 0, None)
torch.cuda.synchronize()
free_setup = torch.cuda.mem_get_info()[0]
ok_1 = round_trip()
torch.cuda.synchronize()
free_1 = torch.cuda.mem_get_info()[0]
ok_2 = all([round_trip() for _ in range(10)])
torch.cuda.synchronize()
free_2 = torch.cuda.mem_get_info()[0]
# take almost all free HBM, then call again
hold = []
while torch.cuda.mem_get_info()[0] > (2 << 30):
    hold.append(torch.empty(1 << 30, dtype=torch.uint8, device="cuda"))
while torch.cuda.mem_get_info()[0] > (192 << 20):
    hold.append(torch.empty(32 << 20, dtype=torch.uint8, device="cuda"))
free_full = torch.cuda.mem_get_info()[0]
ok_full = round_trip()
torch.cuda.synchronize()
free_full_after = torch.cuda.mem_get_info()[0]
del hold
print(json.dumps(dict(setup=setup, free_start=free_start, free_setup=free_setup, free_1=free_1, free_2=free_2,
                      ok_1=ok_1, ok_2=ok_2, free_full=free_full, ok_full=ok_full,
                      free_full_after=free_full_after)))
"""


def test_noalloc_leaves_free_device_memory_unchanged_in_a_fresh_process():
    """In a fresh process: the set-up call (num_records = 0) is where the driver
    may place the static array and the kernels' code in device memory; after
    it, 88 gathers and scatters on both kernel paths take no page of device
    memory, and they still succeed, byte-exact against the golden digests,
    with all but ~192 MiB of the device's free HBM taken."""
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(ROOT / "tests" / "golden" / "kv_records.json")],
                       capture_output=True, text=True, timeout=600, env=env, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["setup"] == 0
    assert res["ok_1"] and res["ok_2"] and res["ok_full"], res
    # Device memory is handed out in 2 MiB pages (cudaMalloc, and the
    # module load the set-up triggers: exactly one page on B200): after the
    # set-up, 88 calls must not take one.  The free bytes normally do not
    # move at all; once, on one box, they dropped by a single 64 KiB step
    # during these calls (not seen again, nor in 400 calls of the entry
    # point alone) -- smaller than anything the library or a module load
    # could take -- so the bound is one page rather than zero.
    page = 2 << 20
    assert res["free_setup"] - res["free_1"] < page, res
    assert res["free_setup"] - res["free_2"] < page, res
    assert res["free_full"] - res["free_full_after"] < page, res
