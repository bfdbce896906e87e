"""vLLM FlashInfer paged layouts on the GPU: the sm_100a gather/scatter
kernel addressing [num_blocks][2][...] blocks, token-major (NHD, bulk and
register paths) and head-major (HND, what vLLM uses on sm_100), against the
golden digests of the reference layout; then the CUDA cache and the
layer-ranged async path with such a cache."""
import ctypes as C

import numpy as np
import pytest
import torch

from demo_b200 import cache as cc
from demo_b200._lib import KVCOPY_ERR_SLOT_RANGE, KVCOPY_FLAG_BULK, KvCopyDesc, lib
from oracle import kvcopy as ok
from tests.flashinfer_layout import as_flash_attn_view, as_vllm_view, from_flashinfer, head_bytes_of, to_flashinfer
from tests.golden import gen
from tests.gpu_util import dsha, ptr_array, to_dev
from tests.test_cache_host import keys_for

pytestmark = pytest.mark.gpu

KV2 = [c for c in gen.KV_CASES if c["kv"] == 2]
GEOMS = [(False, 0), (False, KVCOPY_FLAG_BULK), (True, 0), (True, KVCOPY_FLAG_BULK)]
GEOM_IDS = ["nhd-lsu", "nhd-bulk", "hnd-lsu", "hnd-bulk"]


class FlashInferKV:
    """per-layer FlashInfer tensors of a golden case on the GPU"""

    def __init__(self, case, hnd, zero=False):
        self.case, self.hnd = case, hnd
        k, v = gen.paged_layers(case, zero=zero)
        self.phys = [to_dev(a) for a in to_flashinfer(case, k, v, hnd)]
        half = case["block_size"] * gen.unit_of(case)
        self.kp = torch.tensor([p.data_ptr() for p in self.phys], dtype=torch.int64, device="cuda")
        self.vp = self.kp + half

    def planes(self):
        return from_flashinfer(self.case, [p.cpu().numpy() for p in self.phys], self.hnd)

    def views(self):
        return [as_vllm_view(self.case, p, self.hnd) for p in self.phys]


def launch(kv: FlashInferKV, records, direction, bids=None, slots=None, flags=0, err=None):
    case = kv.case
    recp = ptr_array(records)
    d = KvCopyDesc(layer_k=kv.kp.data_ptr(), layer_v=kv.vp.data_ptr(), records=recp.data_ptr(),
                   slots=slots.data_ptr() if slots is not None else None,
                   block_ids=bids.data_ptr() if bids is not None else None,
                   error=err.data_ptr() if err is not None else None,
                   page_buffer_size=case["num_blocks"] * case["block_size"],
                   unit_bytes=gen.unit_of(case), num_tokens=case["chunk_size"],
                   block_size=case["block_size"], num_layers=case["num_layers"],
                   num_records=len(records), direction=direction, flags=flags,
                   block_stride=2 * case["block_size"] * gen.unit_of(case),
                   head_bytes=head_bytes_of(case) if kv.hnd else 0)
    ret = lib.kv_copy_launch(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return ret


@pytest.mark.parametrize("hnd,flags", GEOMS, ids=GEOM_IDS)
@pytest.mark.parametrize("case", KV2, ids=lambda c: c["name"])
def test_gather_from_flashinfer_gives_reference_records(case, hnd, flags, golden_records):
    kv = FlashInferKV(case, hnd)
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert launch(kv, recs, 1, bids=to_dev(gen.block_ids(case).astype(np.int64)), flags=flags, err=err) == 0
    assert int(err.item()) == 0
    assert [dsha(r) for r in recs] == golden_records[case["name"]]["record_sha256"]


@pytest.mark.parametrize("hnd,flags", GEOMS, ids=GEOM_IDS)
@pytest.mark.parametrize("case", KV2, ids=lambda c: c["name"])
def test_scatter_into_flashinfer_matches_reference_digests(case, hnd, flags, golden_records):
    kv = FlashInferKV(case, hnd, zero=True)
    recs = [to_dev(r) for r in gen.records_for_scatter(case)]
    assert launch(kv, recs, 0, bids=to_dev(gen.block_ids(case, seed_offset=1).astype(np.int64)), flags=flags) == 0
    k, v = kv.planes()
    g = golden_records[case["name"]]
    assert [gen.sha(a) for a in k] == g["scatter_k_sha256"]
    assert [gen.sha(a) for a in v] == g["scatter_v_sha256"]


@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
def test_slot_mode_and_bad_block_on_flashinfer(hnd):
    """per-token slots (a random permutation of the cache's slots) and a
    block id past the cache: the bad block is flagged and the records
    without it are exact"""
    case = next(c for c in KV2 if c["name"] == "gqa_bs16")
    unit, bs, C_ = gen.unit_of(case), case["block_size"], case["chunk_size"]
    kv = FlashInferKV(case, hnd)
    rng = np.random.default_rng(3)
    slots = rng.permutation(case["num_blocks"] * bs)[:C_ * 2].astype(np.int64)
    recs = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(2)]
    assert launch(kv, recs, 1, slots=to_dev(slots)) == 0
    k, v = gen.paged_layers(case)
    for r in range(2):
        e = np.zeros(gen.record_bytes(case), np.uint8)
        ok.transfer(e, k, v, slots[r * C_:(r + 1) * C_], C_, unit, 1, True)
        assert np.array_equal(recs[r].cpu().numpy(), e), r
    bids = gen.block_ids(case).astype(np.int64)
    bad = bids.copy()
    bad[3] = case["num_blocks"]                        # one past the last block
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = [torch.zeros(gen.record_bytes(case), dtype=torch.uint8, device="cuda") for _ in range(case["chunks"])]
    assert launch(kv, out, 1, bids=to_dev(bad), err=err, flags=KVCOPY_FLAG_BULK) == 0
    assert int(err.item()) & KVCOPY_ERR_SLOT_RANGE
    exp = ok.gather(k, v, bids, C_, bs, unit)
    for i in (1, 2):          # records without the bad block are exact
        assert np.array_equal(out[i].cpu().numpy(), exp[i])


@pytest.fixture
def cuda_cache():
    inited = []

    def _init(case, records):
        cc.init(case["chunk_size"], records * gen.record_bytes(case), None)
        inited.append(1)
    yield _init
    if inited:
        cc.exit()


@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
@pytest.mark.parametrize("name", ["gqa_bs16", "tp8_shard"])
def test_cuda_cache_crosses_flash_attn_and_flashinfer(name, hnd, cuda_cache):
    case = next(c for c in KV2 if c["name"] == name)
    unit, bs, C_ = gen.unit_of(case), case["block_size"], case["chunk_size"]
    cuda_cache(case, 2 * case["chunks"] + 1)
    k, v = gen.paged_layers(case)
    fa = [as_flash_attn_view(case, to_dev(a), to_dev(b)) for a, b in zip(k, v)]
    wa = cc.Worker("m", *cc.layout_from_kv_tensors(fa))
    wa.register()
    fi = FlashInferKV(case, hnd, zero=True)
    wf = cc.Worker("m", *cc.layout_from_kv_tensors(fi.views()))
    wf.register()
    keys = keys_for(case["chunks"], seed=21)
    bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
    assert wa.store(keys, bids) == 0
    assert wf.load(keys, b2) == 0
    torch.cuda.synchronize()
    ek, ev = gen.paged_layers(case, zero=True)
    ok.scatter(ok.gather(k, v, bids, C_, bs, unit), ek, ev, b2, C_, bs, unit)
    gk, gv = fi.planes()
    assert all(np.array_equal(a, b) for a, b in zip(gk, ek))
    assert all(np.array_equal(a, b) for a, b in zip(gv, ev))
    wf.unregister()
    wa.unregister()


@pytest.mark.parametrize("hnd", [False, True], ids=["nhd", "hnd"])
def test_layerwise_async_with_flashinfer(hnd, cuda_cache):
    """layer-by-layer store from a FlashInfer cache and layer-by-layer load
    (reverse order, staged through the HBM ring) into another one"""
    case = dict(next(c for c in KV2 if c["name"] == "gqa_bs16"), num_layers=6, num_blocks=128, chunks=6)
    unit, bs, C_ = gen.unit_of(case), case["block_size"], case["chunk_size"]
    cuda_cache(case, case["chunks"] + 1)
    src, dst = FlashInferKV(case, hnd), FlashInferKV(case, hnd, zero=True)
    ws = cc.Worker("m", *cc.layout_from_kv_tensors(src.views()))
    wd = cc.Worker("m", *cc.layout_from_kv_tensors(dst.views()))
    ws.register()
    wd.register()
    keys = keys_for(case["chunks"], seed=22)
    bids, b2 = gen.block_ids(case), gen.block_ids(case, seed_offset=1)
    s = torch.cuda.Stream()
    h = ws.store_async(keys, bids)
    for l in range(case["num_layers"]):
        h.layers(l, l + 1, stream=s)
    assert h.finish() == 0
    h = wd.load_async(keys, b2)
    assert h.records == case["chunks"]
    for l in reversed(range(case["num_layers"])):
        h.layers(l, l + 1, stream=s)
    assert h.finish() == 0
    torch.cuda.synchronize()
    k, v = gen.paged_layers(case)
    ek, ev = gen.paged_layers(case, zero=True)
    ok.scatter(ok.gather(k, v, bids, C_, bs, unit), ek, ev, b2, C_, bs, unit)
    gk, gv = dst.planes()
    assert all(np.array_equal(a, b) for a, b in zip(gk, ek))
    assert all(np.array_equal(a, b) for a, b in zip(gv, ev))
    wd.unregister()
    ws.unregister()
