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
