"""SchedulerAdapter / WorkerAdapter talking to a CrossCache server
(demo_b200.server, or any server of the same protocol) with the reference's
constructor signature (python/adaptor.py:58-291: server_url, zmq context,
model name, world size, kv rank, vLLM block size).

Differences from the reference client: the worker registers 72-byte CUDA IPC
keys (handle + offset, demo_b200.ipc) and K-only caches (MLA) as K-only
(the reference always sends tensor[0] and tensor[1], adaptor.py:152-156);
its node id is the worker's CUDA device, so the TP ranks of one node use
separate server slots (the reference sends 0 from every rank); a store is
sent only after the KV writes queued on the compute stream have finished.
"""
from __future__ import annotations

import threading
from concurrent.futures import Future, ThreadPoolExecutor

import torch

from . import cache as cc
from . import protocol as P
from .adaptor import CHUNK_SIZE, LoadStoreOp, WorkerAdapter, striding_block_hashes
from .ipc import KEY_BYTES, layer_keys
from .mq import MessageQueueClient


class RemoteSchedulerAdapter:
    def __init__(self, server_url: str, context, model_name: str, world_size: int, kv_rank: int,
                 vllm_block_size: int):
        self.mq_client = MessageQueueClient(server_url, context)
        self.instance_id = 0
        self.model_name = model_name
        self.world_size = world_size
        self.worker_id = kv_rank
        self.chunk_size = CHUNK_SIZE
        self.blocks_in_chunk = self.chunk_size // vllm_block_size
        self.lookup_futures: dict[str, Future] = {}

    def try_lookup(self, request_id: str, block_hashes: list[bytes]) -> None:
        if request_id in self.lookup_futures:
            return
        keys = list(striding_block_hashes(block_hashes, self.blocks_in_chunk))
        if not keys:
            fut: Future = Future()
            fut.set_result(0)
        else:
            fut = self.mq_client.submit(lambda uid: P.encode_lookup(
                self.instance_id, uid, keys, self.world_size, self.model_name))
        self.lookup_futures[request_id] = fut

    def check_lookup_result(self, request_id: str) -> int | None:
        """hit tokens, or None while the server has not answered
        (adaptor.py:87-100)"""
        assert request_id in self.lookup_futures, (
            f"Lookup request for request_id={request_id} has not been submitted")
        fut = self.lookup_futures[request_id]
        if not fut.done():
            return None
        return max(0, fut.result())

    def cleanup_lookup_result(self, request_id: str) -> None:
        self.lookup_futures.pop(request_id, None)

    def num_blocks_per_chunk(self) -> int:
        return self.blocks_in_chunk

    def close(self) -> None:
        self.mq_client.close()


class RemoteWorkerAdapter(WorkerAdapter):
    """The worker half; store / load / get_finished bookkeeping as the
    in-process WorkerAdapter, transfers done by the server."""

    def __init__(self, server_url: str, context, model_name: str, world_size: int, kv_rank: int,
                 vllm_block_size: int, device: int | None = None, timeout: float | None = 600.0):
        self.mq_client = MessageQueueClient(server_url, context)
        self.model_name = model_name
        self.world_size = world_size
        self.worker_id = kv_rank
        self.chunk_size = CHUNK_SIZE
        self.blocks_in_chunk = self.chunk_size // vllm_block_size
        self.device = torch.cuda.current_device() if device is None else device
        self.instance_id = self.device
        self.timeout = timeout
        self.tp_group = None
        self.worker = None
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="CrossCacheRemote")
        self.store_futures = {}
        self.load_futures = {}
        self.finished_stores = set()
        self.previously_finished = set()
        self.results = {}
        self.registered = False
        self._failed_load_blocks: set[int] = set()
        self._failed_lock = threading.Lock()

    def register(self, kv_caches: dict[str, torch.Tensor]) -> None:
        tensors = list(kv_caches.values())
        layout, _, _ = cc.layout_from_kv_tensors(tensors)
        kk, vk = layer_keys(tensors)
        per_layer = [(kk[i * KEY_BYTES:(i + 1) * KEY_BYTES],) + (
            (vk[i * KEY_BYTES:(i + 1) * KEY_BYTES],) if vk is not None else ())
            for i in range(layout.num_layers)]
        ret = self.mq_client.request(lambda uid: P.encode_register(
            self.instance_id, uid, self.world_size, self.worker_id, layout.num_blocks, layout.block_size,
            layout.element_size, layout.hidden_dim_size, KEY_BYTES, self.model_name, per_layer,
            layout.block_stride, layout.head_bytes),
            timeout=self.timeout)
        if ret != 0:
            raise cc.CacheError("remote register", ret)
        self.registered = True

    def unregister(self) -> None:
        self._pool.shutdown(wait=True)
        if self.registered:
            self.mq_client.request(lambda uid: P.encode_unregister(self.instance_id, uid),
                                   timeout=self.timeout)
            self.registered = False
        self.mq_client.close()

    def _send(self, op: P.Op, keys: list[bytes], block_ids: list[int]) -> Future:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))

        def run() -> int:
            ev.synchronize()     # the server reads HBM this process wrote
            ret = self.mq_client.request(
                lambda uid: P.encode_transfer(op, self.instance_id, uid, keys, block_ids), timeout=self.timeout)
            if ret and op == P.Op.LOAD:       # one status per message: all its blocks
                with self._failed_lock:
                    self._failed_load_blocks.update(int(b) for b in block_ids)
            return ret
        return self._pool.submit(run)

    def _gather(self, ops: list[LoadStoreOp]) -> tuple[list[bytes], list[int]]:
        """all ops in one message, each trimmed to whole records (the server
        answers -EINVAL when keys and blocks disagree)"""
        keys, block_ids = [], []
        for k, b in zip(*self._per_request(ops)):
            keys.extend(k)
            block_ids.extend(b)
        return keys, block_ids

    def store_requests(self, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        keys, bids = self._gather(ops)
        self.store_futures[request_ids[0]] = (self._send(P.Op.STORE, keys, bids), request_ids[1:])

    def load_requests(self, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        keys, bids = self._gather(ops)
        self.load_futures[request_ids[0]] = (self._send(P.Op.LOAD, keys, bids), request_ids[1:])

    def lookup_agreed(self, keys_per_request):
        raise NotImplementedError("the server answers lookups for rank 0 of the group")
