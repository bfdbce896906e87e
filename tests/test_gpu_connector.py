"""Worker side of the vLLM connector on the GPU: register paged KV tensors,
STORE through wait_for_save, RETRIEVE through start_load_kv, completion
reported by get_finished (CrossCache python/adaptor.py:196-291 semantics),
bytes compared with the source blocks."""
import time
from types import SimpleNamespace

import pytest

pytestmark = pytest.mark.gpu

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")


class _KVT:
    kv_connector_extra_config = {"cache.pool_size": 64 * (2 * 4 * 256 * 8 * 128 * 2)}

    def get_from_extra_config(self, key, default):
        return self.kv_connector_extra_config.get(key, default)


def test_worker_store_then_retrieve_through_connector():
    import torch

    from demo_b200.adaptor import LoadStoreOp
    from demo_b200.connector import CacheConnectorMetadata, CacheRequestMetadata, CrossCacheConnector
    from oracle import blockhash as bh

    cfg = SimpleNamespace(kv_transfer_config=_KVT(), model_config=SimpleNamespace(model="m-gpu"),
                          parallel_config=SimpleNamespace(world_size=1, rank=0),
                          cache_config=SimpleNamespace(block_size=16))
    conn = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.WORKER)
    g = torch.Generator(device="cuda").manual_seed(3)
    kv = {f"layer.{i}": torch.randn(2, 256, 16, 8, 128, generator=g, device="cuda").to(torch.bfloat16)
          for i in range(4)}
    conn.register_kv_caches(kv)
    toks = list(range(1000, 1000 + 1024))
    hashes = bh.block_hashes(toks, 16, bh.none_hash("0"))            # 64 blocks = 4 chunks
    src = list(range(0, 64))
    dst = list(range(100, 164))
    try:
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("R", "STORE", LoadStoreOp(hashes, src)))
        conn.bind_connector_metadata(m)
        conn.wait_for_save()
        conn.clear_connector_metadata()
        deadline = time.time() + 60
        done_s = set()
        while "R" not in done_s and time.time() < deadline:
            s, _ = conn.get_finished({"R"})
            done_s |= s or set()
            time.sleep(0.01)
        assert "R" in done_s
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("R2", "RETRIEVE", LoadStoreOp(hashes, dst)))
        conn.bind_connector_metadata(m)
        conn.start_load_kv(None)
        conn.clear_connector_metadata()
        done_l = set()
        while "R2" not in done_l and time.time() < deadline:
            _, l = conn.get_finished(set())
            done_l |= l or set()
            time.sleep(0.01)
        assert "R2" in done_l
        assert conn.worker_adapter.wait_all(timeout=10) == []
        assert conn.worker_adapter.results == {"R": 0, "R2": 0}
        torch.cuda.synchronize()
        for t in kv.values():
            assert torch.equal(t[:, src].view(torch.int16), t[:, dst].view(torch.int16))
    finally:
        conn.shutdown()


def test_layerwise_worker_steps():
    """cache.layerwise: a step whose "attention" rewrites each layer after a
    delay and calls save_kv_layer, then a step that loads the chunks back
    layer by layer while its "attention" reads each layer after
    wait_for_layer_load -- both orderings enforced on the GPU only"""
    import torch

    from demo_b200.adaptor import LoadStoreOp
    from demo_b200.connector import CacheConnectorMetadata, CacheRequestMetadata, CrossCacheConnector
    from oracle import blockhash as bh

    kvt = _KVT()
    kvt.kv_connector_extra_config = dict(_KVT.kv_connector_extra_config, **{"cache.layerwise": True})
    cfg = SimpleNamespace(kv_transfer_config=kvt, model_config=SimpleNamespace(model="m-layerwise"),
                          parallel_config=SimpleNamespace(world_size=1, rank=0),
                          cache_config=SimpleNamespace(block_size=16))
    conn = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.WORKER)
    g = torch.Generator(device="cuda").manual_seed(5)
    kv = {f"model.layers.{i}.attn": torch.zeros(2, 256, 16, 8, 128, device="cuda", dtype=torch.bfloat16)
          for i in range(4)}
    new = {n: torch.randn(2, 64, 16, 8, 128, generator=g, device="cuda").to(torch.bfloat16) for n in kv}
    conn.register_kv_caches(kv)
    toks = list(range(5000, 5000 + 1024))
    hashes = bh.block_hashes(toks, 16, bh.none_hash("0"))
    src, dst = list(range(0, 64)), list(range(100, 164))
    src_t = torch.tensor(src, device="cuda")
    dst_t = torch.tensor(dst, device="cuda")
    try:
        # step 1: the forward writes each layer late; the save must wait for it
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("S", "STORE", LoadStoreOp(hashes, src)))
        conn.bind_connector_metadata(m)
        conn.start_load_kv(None)
        for name, t in kv.items():
            conn.wait_for_layer_load(name)
            torch.cuda._sleep(5_000_000)
            t[:, src_t] = new[name]
            conn.save_kv_layer(name, t, None)
        conn.wait_for_save()
        conn.clear_connector_metadata()
        deadline = time.time() + 60
        done = set()
        while "S" not in done and time.time() < deadline:
            s, _ = conn.get_finished({"S"})
            done |= s or set()
            time.sleep(0.01)
        assert "S" in done and conn.worker_adapter.results["S"] == 0
        # step 2: load into other blocks; each layer is read right after its wait
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("L", "RETRIEVE", LoadStoreOp(hashes, dst)))
        conn.bind_connector_metadata(m)
        conn.start_load_kv(None)
        seen = {}
        for name, t in kv.items():
            conn.wait_for_layer_load(name)
            seen[name] = t[:, dst_t].clone()
            conn.save_kv_layer(name, t, None)
        conn.wait_for_save()
        conn.clear_connector_metadata()
        _, loads = conn.get_finished(set())
        assert not loads                       # synchronous loads are not reported
        torch.cuda.synchronize()
        for name in kv:
            assert torch.equal(seen[name].view(torch.int16), new[name].view(torch.int16)), name
            assert torch.equal(kv[name][:, dst_t].view(torch.int16), new[name].view(torch.int16)), name
    finally:
        conn.shutdown()


def test_failed_loads_are_reported_per_request():
    """two requests in one RETRIEVE step, one of them never stored: it alone
    fails, and its blocks come back from get_block_ids_with_load_errors"""
    import torch

    from demo_b200.adaptor import LoadStoreOp
    from demo_b200.connector import CacheConnectorMetadata, CacheRequestMetadata, CrossCacheConnector
    from oracle import blockhash as bh

    cfg = SimpleNamespace(kv_transfer_config=_KVT(), model_config=SimpleNamespace(model="m-errors"),
                          parallel_config=SimpleNamespace(world_size=1, rank=0),
                          cache_config=SimpleNamespace(block_size=16))
    conn = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.WORKER)
    kv = {f"layer.{i}": torch.randn(2, 256, 16, 8, 128, device="cuda").to(torch.bfloat16) for i in range(4)}
    conn.register_kv_caches(kv)
    good = bh.block_hashes(list(range(100, 100 + 512)), 16, bh.none_hash("0"))     # 32 blocks
    bad = bh.block_hashes(list(range(900, 900 + 512)), 16, bh.none_hash("0"))
    try:
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("G", "STORE", LoadStoreOp(good, list(range(32)))))
        conn.bind_connector_metadata(m)
        conn.wait_for_save()
        conn.clear_connector_metadata()
        assert conn.worker_adapter.wait_all(timeout=60) == [0]
        m = CacheConnectorMetadata()
        m.add_request_metadata(CacheRequestMetadata("LG", "RETRIEVE", LoadStoreOp(good, list(range(100, 132)))))
        m.add_request_metadata(CacheRequestMetadata("LB", "RETRIEVE", LoadStoreOp(bad, list(range(140, 172)))))
        conn.bind_connector_metadata(m)
        conn.start_load_kv(None)
        conn.clear_connector_metadata()
        deadline = time.time() + 60
        done = set()
        while done != {"LG", "LB"} and time.time() < deadline:
            _, l = conn.get_finished(set())
            done |= l or set()
            time.sleep(0.01)
        assert done == {"LG", "LB"}
        assert conn.get_block_ids_with_load_errors() == set(range(140, 172))
        assert conn.get_block_ids_with_load_errors() == set()
        res = conn.worker_adapter.results
        assert res["G"] == 0 and res["LG"] == 0 and res["LB"] == -2
        torch.cuda.synchronize()
        for t in kv.values():
            assert torch.equal(t[:, 0:32].view(torch.int16), t[:, 100:132].view(torch.int16))
    finally:
        conn.shutdown()
