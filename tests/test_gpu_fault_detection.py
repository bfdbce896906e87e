"""Failure detection inside the TMA bulk kernels, without a GPU fault.

Every mbarrier wait of kv_copy_bulk_kernel and kv_copy_bulk_hnd_kernel is
bounded: when it runs out the kernel sets KVCOPY_ERR_TIMEOUT, waits (with one
bounded budget) for its other loads in flight, and returns, so the host reads
an error status and the context stays usable.  KVCOPY_FLAG_TEST_STALL makes
CTA 0 arm its first stage's barrier for 16 bytes that it never copies: that
wait runs out after a few milliseconds with no copy in flight on the stage
(nothing is left writing shared memory when the CTA exits).  Each test
checks the error bit, that the call returned promptly, and that the next
launch on the same context gives the golden mem.cpp bytes."""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from demo_b200._lib import (KVCOPY_ERR_TIMEOUT, KVCOPY_FLAG_BULK, KVCOPY_FLAG_TEST_STALL, KVCOPY_PATH_BULK,
                            KVCOPY_PATH_BULK_HND, KvCopyDesc, lib)
from tests.flashinfer_layout import from_flashinfer, head_bytes_of, to_flashinfer
from tests.golden import gen
from tests.gpu_util import DeviceKV, dsha, ptr_array, to_dev

pytestmark = pytest.mark.gpu

CASE = next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16")   # 32 KiB block runs: bulk path


def _desc(kp, vp, recs, bids, err, direction, flags, block_stride=0, head_bytes=0):
    c = CASE
    return KvCopyDesc(layer_k=kp.data_ptr(), layer_v=vp.data_ptr(), records=ptr_array(recs).data_ptr(),
                      slots=None, block_ids=bids.data_ptr(), error=err.data_ptr(),
                      page_buffer_size=c["num_blocks"] * c["block_size"], unit_bytes=gen.unit_of(c),
                      num_tokens=c["chunk_size"], block_size=c["block_size"], num_layers=c["num_layers"],
                      num_records=len(recs), direction=direction, flags=flags, block_stride=block_stride,
                      head_bytes=head_bytes)


def _run(d, keep):
    """launch on the current stream; (return code, error word, seconds)"""
    err = keep
    err.zero_()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ret = lib.kv_copy_launch(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return ret, int(err.item()), time.perf_counter() - t0


@pytest.mark.parametrize("direction", [1, 0], ids=["gather", "scatter"])
def test_bulk_kernel_wait_runs_out_then_next_launch_is_exact(direction, golden_records):
    g = golden_records[CASE["name"]]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kv = DeviceKV(CASE, zero=(direction == 0))
    if direction:
        recs = [torch.zeros(gen.record_bytes(CASE), dtype=torch.uint8, device="cuda") for _ in range(CASE["chunks"])]
        bids = to_dev(gen.block_ids(CASE).astype(np.int64))
    else:
        recs = [to_dev(r) for r in gen.records_for_scatter(CASE)]
        bids = to_dev(gen.block_ids(CASE, seed_offset=1).astype(np.int64))
    stalled = _desc(kv.kp, kv.vp, recs, bids, err, direction, KVCOPY_FLAG_BULK | KVCOPY_FLAG_TEST_STALL)
    assert lib.kv_copy_path(C.byref(stalled)) == KVCOPY_PATH_BULK
    ret, bits, secs = _run(stalled, err)
    assert ret == 0                                   # the launch itself succeeded
    assert bits & KVCOPY_ERR_TIMEOUT, bits            # the kernel reported the wait that ran out
    assert secs < 1.0, secs                           # and returned on its own, promptly
    # the context is usable: the same transfer without the flag is exact
    ret, bits, _ = _run(_desc(kv.kp, kv.vp, recs, bids, err, direction, KVCOPY_FLAG_BULK), err)
    assert ret == 0 and bits == 0
    if direction:
        assert [dsha(r) for r in recs] == g["record_sha256"]
    else:
        assert [dsha(t) for t in kv.k] == g["scatter_k_sha256"]
        assert [dsha(t) for t in kv.v] == g["scatter_v_sha256"]


@pytest.mark.parametrize("direction", [1, 0], ids=["gather", "scatter"])
def test_head_major_bulk_kernel_wait_runs_out_then_next_launch_is_exact(direction, golden_records):
    """the same for vLLM FlashInfer's head-major blocks (the transposing kernel,
    whose 512 threads follow thread 0's bounded wait through a CTA barrier)"""
    g = golden_records[CASE["name"]]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    k, v = gen.paged_layers(CASE, zero=(direction == 0))
    phys = [to_dev(a) for a in to_flashinfer(CASE, k, v, True)]
    kp = torch.tensor([p.data_ptr() for p in phys], dtype=torch.int64, device="cuda")
    vp = kp + CASE["block_size"] * gen.unit_of(CASE)
    stride, hb = 2 * CASE["block_size"] * gen.unit_of(CASE), head_bytes_of(CASE)
    if direction:
        recs = [torch.zeros(gen.record_bytes(CASE), dtype=torch.uint8, device="cuda") for _ in range(CASE["chunks"])]
        bids = to_dev(gen.block_ids(CASE).astype(np.int64))
    else:
        recs = [to_dev(r) for r in gen.records_for_scatter(CASE)]
        bids = to_dev(gen.block_ids(CASE, seed_offset=1).astype(np.int64))
    stalled = _desc(kp, vp, recs, bids, err, direction, KVCOPY_FLAG_BULK | KVCOPY_FLAG_TEST_STALL, stride, hb)
    assert lib.kv_copy_path(C.byref(stalled)) == KVCOPY_PATH_BULK_HND
    ret, bits, secs = _run(stalled, err)
    assert ret == 0 and bits & KVCOPY_ERR_TIMEOUT and secs < 1.0, (ret, bits, secs)
    ret, bits, _ = _run(_desc(kp, vp, recs, bids, err, direction, KVCOPY_FLAG_BULK, stride, hb), err)
    assert ret == 0 and bits == 0
    if direction:
        assert [dsha(r) for r in recs] == g["record_sha256"]
    else:
        kk, vv = from_flashinfer(CASE, [p.cpu().numpy() for p in phys], True)
        assert [gen.sha(a) for a in kk] == g["scatter_k_sha256"]
        assert [gen.sha(a) for a in vv] == g["scatter_v_sha256"]


def test_stall_flag_is_ignored_by_the_register_path_and_unknown_flags_are_rejected():
    """the register kernel waits on nothing: the flag changes nothing there;
    bits outside the defined flags make the descriptor invalid"""
    import errno
    tp8 = next(c for c in gen.KV_CASES if c["name"] == "tp8_shard")
    kv = DeviceKV(tp8)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    recs = [torch.zeros(gen.record_bytes(tp8), dtype=torch.uint8, device="cuda") for _ in range(tp8["chunks"])]
    bids = to_dev(gen.block_ids(tp8).astype(np.int64))
    d = KvCopyDesc(layer_k=kv.kp.data_ptr(), layer_v=kv.vp.data_ptr(), records=ptr_array(recs).data_ptr(),
                   slots=None, block_ids=bids.data_ptr(), error=err.data_ptr(),
                   page_buffer_size=tp8["num_blocks"] * tp8["block_size"], unit_bytes=gen.unit_of(tp8),
                   num_tokens=tp8["chunk_size"], block_size=tp8["block_size"], num_layers=tp8["num_layers"],
                   num_records=len(recs), direction=1, flags=KVCOPY_FLAG_BULK | KVCOPY_FLAG_TEST_STALL)
    ret, bits, _ = _run(d, err)
    assert ret == 0 and bits == 0
    d.flags = 0x40
    assert lib.kv_copy_launch(C.byref(d), None) == -errno.EINVAL
    assert lib.kv_copy_path(C.byref(d)) == -errno.EINVAL
