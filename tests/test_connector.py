"""Scheduler side of the vLLM connector (CrossCacheConnector) against an
in-process cache on the explicit CPU backend: lookup -> matched tokens,
tracker states, and the chunk-granular STORE / RETRIEVE metadata of
CrossCache's python/crosscache_connector.py:205-294, 490-661."""
from types import SimpleNamespace

import numpy as np
import pytest

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")

from demo_b200 import cache as cc  # noqa: E402
from demo_b200._lib import CACHE_BACKEND_MEM  # noqa: E402
from demo_b200.connector import (CacheConnectorMetadata, CacheRequestState,  # noqa: E402
                                 CrossCacheConnector)
from oracle import blockhash as bh  # noqa: E402

BS = 16


class _KVT:
    def __init__(self):
        self.kv_connector_extra_config = {}

    def get_from_extra_config(self, key, default):
        return self.kv_connector_extra_config.get(key, default)


def _cfg():
    return SimpleNamespace(kv_transfer_config=_KVT(), model_config=SimpleNamespace(model="m"),
                           parallel_config=SimpleNamespace(world_size=1, rank=0),
                           cache_config=SimpleNamespace(block_size=BS))


def _request(rid, ntok, seed):
    toks = np.random.default_rng(seed).integers(0, 128256, ntok).tolist()
    return SimpleNamespace(request_id=rid, all_token_ids=toks, num_tokens=ntok,
                           block_hashes=bh.block_hashes(toks, BS, bh.none_hash("0")))


class _Blocks:
    def __init__(self, ids):
        self.ids = list(ids)

    def get_block_ids(self):
        return (self.ids,)


def _sched_out(new=(), cached=None):
    cached = cached or SimpleNamespace(req_ids=[], new_block_ids=[], num_computed_tokens=[])
    return SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(req_id=r) for r, _ in new],
                           num_scheduled_tokens={r: n for r, n in new}, scheduled_cached_reqs=cached)


@pytest.fixture
def sched():
    # a MEM-backend worker of model "m" holding the stored chunks
    nb, unit = 256, 64
    layers = [np.zeros(nb * BS * unit, np.uint8) for _ in range(2)]
    cc.init(256, 8 * 2 * 1 * 256 * unit, None, CACHE_BACKEND_MEM)
    lay = cc.KVLayout(1, nb, BS, 32, 2, 2)
    w = cc.Worker("m", lay, [layers[0].ctypes.data], [layers[1].ctypes.data])
    w.register()
    conn = CrossCacheConnector(_cfg(), vllm_base.KVConnectorRole.SCHEDULER)
    conn.scheduler_adapter.bind_worker(w)
    yield conn, w
    w.unregister()
    cc.exit()


def test_lookup_alloc_and_retrieve_store_metadata(sched):
    conn, w = sched
    req = _request("A", 1024, 1)                     # 64 blocks = 4 chunks
    keys = bh.chunk_keys(req.block_hashes, 256 // BS)
    assert w.store(keys[:2], np.arange(32)) == 0    # first 2 chunks cached
    n, load_async = conn.get_num_new_matched_tokens(req, 0)
    assert (n, load_async) == (512, True)
    conn.update_state_after_alloc(req, _Blocks(range(100, 164)), 512)
    t = conn.request_trackers["A"]
    assert t.state == CacheRequestState.WAITING_FOR_LOAD
    assert (t.num_vllm_hit_blocks, t.num_cache_hit_blocks, t.num_stored_blocks) == (0, 32, 32)
    meta = conn.build_connector_meta(_sched_out(new=[("A", 1024)]))
    assert isinstance(meta, CacheConnectorMetadata)
    kinds = [(m.direction, len(m.op)) for m in meta.requests]
    assert kinds == [("RETRIEVE", 32), ("STORE", 32)]
    ret, store = meta.requests
    assert ret.op.block_ids == list(range(100, 132))
    assert ret.op.block_hashes == req.block_hashes[:32]
    assert store.op.block_ids == list(range(132, 164))
    assert store.op.block_hashes == req.block_hashes[32:64]
    assert t.state == CacheRequestState.READY
    assert conn.request_finished(req, []) == (True, None)
    assert "A" not in conn.request_trackers


def test_partial_vllm_hit_retrieves_from_chunk_boundary(sched):
    conn, w = sched
    req = _request("B", 1024, 2)
    keys = bh.chunk_keys(req.block_hashes, 256 // BS)
    assert w.store(keys[:3], np.arange(48)) == 0     # 3 chunks cached = 48 blocks
    # vLLM already holds 20 blocks (320 tokens): load from chunk 1 (block 16)
    n, load_async = conn.get_num_new_matched_tokens(req, 320)
    assert (n, load_async) == (768 - 320, True)
    conn.update_state_after_alloc(req, _Blocks(range(64)), 448)
    meta = conn.build_connector_meta(_sched_out())
    (ret,) = meta.requests
    assert ret.direction == "RETRIEVE"
    assert ret.op.block_ids == list(range(16, 48))
    assert ret.op.block_hashes == req.block_hashes[16:48]


def test_miss_goes_ready_and_stores_whole_chunks_only(sched):
    conn, _ = sched
    req = _request("C", 700, 3)                      # 43 full blocks
    assert conn.get_num_new_matched_tokens(req, 0) == (0, False)
    conn.update_state_after_alloc(req, _Blocks(range(10, 54)), 0)
    assert conn.request_trackers["C"].state == CacheRequestState.READY
    # 600 tokens scheduled -> 37 full blocks -> 2 whole chunks (32 blocks) stored
    meta = conn.build_connector_meta(_sched_out(new=[("C", 600)]))
    (st,) = meta.requests
    assert st.direction == "STORE" and st.op.block_ids == list(range(10, 42))
    # next step: a cached-request update adds tokens; no new whole chunk yet
    cached = SimpleNamespace(req_ids=["C"], new_block_ids=[None], num_computed_tokens=[100])
    meta2 = conn.build_connector_meta(_sched_out(cached=cached))
    assert len(meta2) == 0


def test_unbound_scheduler_reports_no_hits():
    conn = CrossCacheConnector(_cfg(), vllm_base.KVConnectorRole.SCHEDULER)
    req = _request("D", 512, 4)
    assert conn.get_num_new_matched_tokens(req, 0) == (0, False)


def test_remote_scheduler_asks_the_server():
    """cache.server.host / port set: the scheduler's lookups go to a CrossCache
    server over ZeroMQ (the reference connector's deployment), answered from
    the records a worker stored there"""
    import struct
    import time

    pytest.importorskip("zmq")
    from demo_b200 import protocol as P
    from demo_b200.mq import MessageQueueClient
    from demo_b200.server import CacheServer

    nb, unit = 256, 64
    layers = [np.zeros(nb * BS * unit, np.uint8) for _ in range(2)]
    srv = CacheServer("tcp://127.0.0.1:*", 256, 8 * 2 * 256 * unit, None, CACHE_BACKEND_MEM).start()
    cli = MessageQueueClient(srv.endpoint)
    conn = None
    try:
        keys_raw = [(struct.pack("<Q", layers[0].ctypes.data), struct.pack("<Q", layers[1].ctypes.data))]
        assert cli.request(lambda u: P.encode_register(0, u, 1, 0, nb, BS, 2, 32, 8, "m", keys_raw),
                           timeout=30) == 0
        req = _request("R", 1024, 5)
        keys = bh.chunk_keys(req.block_hashes, 256 // BS)
        assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys[:3], list(range(48))),
                           timeout=30) == 0
        cfg = _cfg()
        host, port = srv.endpoint.rsplit(":", 1)
        host = host.split("://", 1)[1]       # a bare host: the connector adds tcp://
        cfg.kv_transfer_config.kv_connector_extra_config.update({"cache.server.host": host,
                                                                 "cache.server.port": int(port)})
        conn = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.SCHEDULER)
        deadline = time.time() + 30
        while (res := conn.get_num_new_matched_tokens(req, 0)) == (None, True) and time.time() < deadline:
            time.sleep(0.01)                 # the answer is asynchronous, as in the reference
        assert res == (768, True)
        conn.update_state_after_alloc(req, _Blocks(range(100, 164)), 768)
        meta = conn.build_connector_meta(_sched_out())
        (ret,) = meta.requests
        assert ret.direction == "RETRIEVE" and ret.op.block_ids == list(range(100, 148))
    finally:
        if conn is not None:
            conn.shutdown()
        cli.close()
        srv.stop()


def test_layerwise_scheduler_loads_inside_the_step(sched):
    """cache.layerwise: hits are loaded synchronously (load_async False)"""
    conn, w = sched
    cfg = _cfg()
    cfg.kv_transfer_config.kv_connector_extra_config["cache.layerwise"] = True
    lw = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.SCHEDULER)
    lw.scheduler_adapter.bind_worker(w)
    req = _request("LW", 1024, 6)
    keys = bh.chunk_keys(req.block_hashes, 256 // BS)
    assert w.store(keys[:2], np.arange(32)) == 0
    assert lw.get_num_new_matched_tokens(req, 0) == (512, False)
    lw.update_state_after_alloc(req, _Blocks(range(64)), 512)
    meta = lw.build_connector_meta(_sched_out(new=[("LW", 1024)]))
    assert [m.direction for m in meta.requests] == ["RETRIEVE", "STORE"]


def test_layerwise_full_prompt_hit_leaves_the_last_token_to_compute(sched):
    """every chunk of a 1024-token prompt cached: the in-step load may not
    cover the whole prompt (vLLM's scheduler needs a token to compute), so
    layer-wise answers 1023; the asynchronous mode answers 1024 and vLLM
    trims it itself.  The load still covers all four records."""
    conn, w = sched
    cfg = _cfg()
    cfg.kv_transfer_config.kv_connector_extra_config["cache.layerwise"] = True
    lw = CrossCacheConnector(cfg, vllm_base.KVConnectorRole.SCHEDULER)
    lw.scheduler_adapter.bind_worker(w)
    req = _request("FULL", 1024, 11)
    keys = bh.chunk_keys(req.block_hashes, 256 // BS)
    assert w.store(keys, np.arange(64)) == 0
    assert lw.get_num_new_matched_tokens(req, 0) == (1023, False)
    lw.update_state_after_alloc(req, _Blocks(range(100, 164)), 1023)
    meta = lw.build_connector_meta(_sched_out(new=[("FULL", 1024)]))
    ret = [m for m in meta.requests if m.direction == "RETRIEVE"]
    assert len(ret) == 1 and ret[0].op.block_ids == list(range(100, 164))
    req2 = _request("FULL", 1024, 11)
    req2.request_id = "FULL-async"
    assert conn.get_num_new_matched_tokens(req2, 0) == (1024, True)


def test_xxhash_block_hashes_become_32_byte_keys(sched):
    """vLLM configured with xxhash (16-byte digests): the connector stores
    and finds the records under zero-padded 32-byte keys"""
    from demo_b200.adaptor import cache_key

    conn, w = sched
    rng = np.random.default_rng(9)
    hashes = [rng.integers(0, 256, 16, dtype=np.uint8).tobytes() for _ in range(64)]
    req = _request("X", 1024, 7)
    req.block_hashes = hashes
    keys = [cache_key(h) for h in hashes[15::16]]
    assert all(len(k) == 32 and k[16:] == bytes(16) for k in keys)
    assert w.store(keys[:3], np.arange(48)) == 0
    assert conn.get_num_new_matched_tokens(req, 0) == (768, True)
    with pytest.raises(ValueError):
        cache_key(bytes(48))
