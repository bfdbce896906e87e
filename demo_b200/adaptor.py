"""SchedulerAdapter / WorkerAdapter with the interface of CrossCache's
python/adaptor.py:43-291, running the cache manager in-process.

The reference adapters serialise every call into ZeroMQ messages for the C
server (register / lookup / store / load, python/utils/protocol.py) and wait
on futures.  Here the same calls go straight to the C API of
libcrosscache.so: lookups answer immediately, stores and loads run on a
worker thread so that wait_for_save / start_load_kv return at once and
get_finished reports completion, exactly as the reference's futures do.
"""
from __future__ import annotations

import logging
import os
import threading
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from itertools import islice
from typing import Iterable

import numpy as np
import torch

from . import cache as cc
from .tp import agree_min_hits

CHUNK_SIZE = 256          # tokens per record (python/adaptor.py:74,133)
logger = logging.getLogger(__name__)

_service_lock = threading.Lock()
_service_refs = 0


def ensure_cache(pool_size: int, chunk_size: int = CHUNK_SIZE, cache_dir: str | None = None) -> None:
    """Process-wide cache_init on first use (the reference's server does
    cache_init once at start-up, src/main.c:388-413).  The disk tier's
    directory is `cache_dir`, else $CROSSCACHE_CACHEDIR (the reference
    server's --cachedir, main.c:436-448); neither means memory only."""
    global _service_refs
    with _service_lock:
        if _service_refs == 0:
            cc.init(chunk_size, pool_size, cache_dir or os.getenv("CROSSCACHE_CACHEDIR") or None)
        _service_refs += 1


def release_cache() -> None:
    global _service_refs
    with _service_lock:
        _service_refs -= 1
        if _service_refs == 0:
            cc.exit()


def cache_key(block_hash: bytes) -> bytes:
    """The 32-byte record key of a vLLM block hash.  sha256 / sha256_cbor
    hashes are 32 bytes and used as they are; xxhash / xxhash_cbor give 16
    (vllm/utils/hashing.py xxh3_128), which the reference's 32-byte key
    compare (src/cache/cache.c:139-145) cannot take: they are zero-padded,
    which keeps distinct digests distinct.  Longer hashes are rejected."""
    b = bytes(block_hash)
    if len(b) == 32:
        return b
    if len(b) < 32:
        return b + bytes(32 - len(b))
    raise ValueError(f"block hash of {len(b)} bytes: keys are 32 bytes")


def striding_block_hashes(block_hashes: list[bytes], blocks_in_chunk: int) -> Iterable[bytes]:
    """Keys of blocks blocks_in_chunk-1, 2*blocks_in_chunk-1, ...
    (python/adaptor.py:32-40): one key per 256-token record."""
    return (cache_key(h) for h in islice(block_hashes, blocks_in_chunk - 1, None, blocks_in_chunk))


@dataclass
class LoadStoreOp:
    block_hashes: list[bytes]
    block_ids: list[int]

    def __len__(self) -> int:
        return len(self.block_hashes)

    def __post_init__(self):
        assert len(self.block_hashes) == len(self.block_ids), (
            "The number of block hashes should be equal to the number of block ids "
            f"But got {len(self.block_hashes)} and {len(self.block_ids)}")


class SchedulerAdapter:
    """python/adaptor.py:58-114.  try_lookup / check_lookup_result give the
    number of cached tokens of a request's prefix (hit records x 256)."""

    def __init__(self, model_name: str, world_size: int, kv_rank: int, vllm_block_size: int,
                 lookup_worker: "cc.Worker | None" = None):
        self.model_name = model_name
        self.world_size = world_size
        self.worker_id = kv_rank
        self.chunk_size = CHUNK_SIZE
        self.blocks_in_chunk = self.chunk_size // vllm_block_size
        self.lookup_results: dict[str, int] = {}
        self._worker = lookup_worker

    def bind_worker(self, worker: "cc.Worker") -> None:
        self._worker = worker

    def try_lookup(self, request_id: str, block_hashes: list[bytes]) -> None:
        if request_id in self.lookup_results:
            return
        keys = list(striding_block_hashes(block_hashes, self.blocks_in_chunk))
        if self._worker is None or not keys:
            self.lookup_results[request_id] = 0
            return
        hit_bytes = self._worker.lookup(keys)
        # src/main.c:140: (hit bytes / key_len) * chunk_size tokens
        self.lookup_results[request_id] = (hit_bytes // cc.KEY_LEN) * self.chunk_size

    def check_lookup_result(self, request_id: str) -> int | None:
        assert request_id in self.lookup_results, (
            f"Lookup request for request_id={request_id} has not been submitted")
        return self.lookup_results[request_id]

    def cleanup_lookup_result(self, request_id: str) -> None:
        self.lookup_results.pop(request_id, None)

    def num_blocks_per_chunk(self) -> int:
        return self.blocks_in_chunk


class WorkerAdapter:
    """python/adaptor.py:117-291 with the same store/load/get_finished
    bookkeeping; the transfers run in this process, stores and loads each on
    a worker thread of their own."""

    def __init__(self, model_name: str, world_size: int, kv_rank: int, vllm_block_size: int,
                 pool_size: int = 4 << 30, device: int | None = None, tp_group=None):
        self.model_name = model_name
        self.world_size = world_size
        self.worker_id = kv_rank
        self.chunk_size = CHUNK_SIZE
        self.blocks_in_chunk = self.chunk_size // vllm_block_size
        self.pool_size = pool_size
        self.device = torch.cuda.current_device() if device is None else device
        self.tp_group = tp_group
        self.worker: cc.Worker | None = None
        # one thread per direction, like the reference server's separate Store
        # and Load pools (src/main.c:394-410): a step's loads do not queue
        # behind the previous step's stores, and the host link carries both
        # directions at once; each direction keeps its submission order
        self._store_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="CrossCacheStore")
        self._load_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="CrossCacheLoad")
        self.store_futures: dict[str, tuple[Future, list[str]]] = {}
        self.load_futures: dict[str, tuple[Future, list[str]]] = {}
        self.finished_stores: set[str] = set()
        self.previously_finished: set[str] = set()
        self.results: dict[str, int] = {}      # return code of each finished store/load, by request
        # layer-wise mode (connector "cache.layerwise"): per-step async handles
        self.layer_index: dict[str, int] = {}
        self._load_stream = None
        self._save_stream = None
        self._layer_load: "cc.AsyncTransfer | None" = None
        self._layer_store: "cc.AsyncTransfer | None" = None
        self._layer_store_ids: list[str] = []
        self._layer_load_futures: list[Future] = []
        self._failed_load_blocks: set[int] = set()
        self._failed_lock = threading.Lock()

    def _block_hashes_to_keys(self, block_hashes: list[bytes]) -> list[bytes]:
        return list(striding_block_hashes(block_hashes, self.blocks_in_chunk))

    def register(self, kv_caches: dict[str, torch.Tensor]) -> None:
        self.layer_index = {name: i for i, name in enumerate(kv_caches)}
        layout, kp, vp = cc.layout_from_kv_tensors(kv_caches.values())
        ensure_cache(self.pool_size)
        self.worker = cc.Worker(self.model_name, layout, kp, vp, node_id=self.device,
                                world_size=self.world_size, rank=self.worker_id)
        self.worker.register()

    def unregister(self) -> None:
        self.end_layerwise_step()
        self._store_pool.shutdown(wait=True)
        self._load_pool.shutdown(wait=True)
        if self.worker is not None:
            self.worker.unregister()
            self.worker = None
            release_cache()

    def _submit(self, pool: ThreadPoolExecutor, fn, *args) -> Future:
        # the transfer must see every KV write queued on the compute stream
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))

        def run():
            ev.synchronize()
            return fn(*args)
        return pool.submit(run)

    def _per_request(self, ops: list[LoadStoreOp]) -> tuple[list[list[bytes]], list[list[int]]]:
        kreq = [list(self._block_hashes_to_keys(op.block_hashes)) for op in ops]
        # whole records only (cache_op ignores a trailing partial chunk too)
        breq = [list(op.block_ids[:len(k) * self.blocks_in_chunk]) for op, k in zip(ops, kreq)]
        return kreq, breq

    def store_requests(self, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        kreq, breq = self._per_request(ops)

        def run():
            ret, st = self.worker.store_batch(kreq, breq)
            return ret, {rid: int(s) for rid, s in zip(request_ids, st)}
        self.store_futures[request_ids[0]] = (self._submit(self._store_pool, run), request_ids[1:])

    def load_requests(self, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        kreq, breq = self._per_request(ops)

        def run():
            ret, st = self.worker.load_batch(kreq, breq)
            failed = [b for s, b in zip(st, breq) if s]
            if failed:
                with self._failed_lock:
                    for b in failed:
                        self._failed_load_blocks.update(int(x) for x in b)
            return ret, {rid: int(s) for rid, s in zip(request_ids, st)}
        self.load_futures[request_ids[0]] = (self._submit(self._load_pool, run), request_ids[1:])

    def take_failed_load_blocks(self) -> set[int]:
        """block ids whose load failed since the last call (for vLLM's
        get_block_ids_with_load_errors: recompute them instead)"""
        with self._failed_lock:
            out, self._failed_load_blocks = self._failed_load_blocks, set()
        return out

    # ---- layer-wise transfers -------------------------------------------
    # The load of a step runs layer by layer on a side stream while the
    # forward pass runs; wait_layer makes the compute stream wait, on the
    # GPU, for one layer.  The store of a step gathers each layer right after
    # the forward wrote it (save_layer), on another side stream, gated on an
    # event of the compute stream; end_layerwise_step hands the store to the
    # worker thread, whose completion get_finished reports as for store_requests.
    def _streams(self):
        if self._load_stream is None:
            self._load_stream = torch.cuda.Stream(self.device)
            self._save_stream = torch.cuda.Stream(self.device)

    def begin_layerwise_load(self, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        keys, block_ids = [], []
        for op in ops:
            keys.extend(self._block_hashes_to_keys(op.block_hashes))
            block_ids.extend(op.block_ids)
        if not keys:
            return
        self._streams()
        # blocks handed to this load may have been read by kernels still queued
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        h = self.worker.load_async(keys, block_ids)
        if h.missing:
            # sync loads report failures in the pass that finds them: the
            # blocks of this step's loads are recomputed
            logger.error("Layer-wise load for %s: some records are no longer cached", request_ids)
            with self._failed_lock:
                self._failed_load_blocks.update(int(b) for b in block_ids)
        for l in range(self.worker.layout.num_layers):
            h.layers(l, l + 1, stream=self._load_stream, wait_event=ready if l == 0 else None)
        self._layer_load = h

    def wait_layer(self, layer_name: str) -> None:
        if self._layer_load is not None:
            self._layer_load.stream_wait(self.layer_index[layer_name], torch.cuda.current_stream(self.device))

    def save_layer(self, layer_name: str, request_ids: list[str], ops: list[LoadStoreOp]) -> None:
        if self._layer_store is None:
            keys, block_ids = [], []
            for op in ops:
                keys.extend(self._block_hashes_to_keys(op.block_hashes))
                block_ids.extend(op.block_ids)
            if not keys:
                return
            self._streams()
            self._layer_store = self.worker.store_async(keys, block_ids)
            self._layer_store_ids = list(request_ids)
        written = torch.cuda.Event()
        written.record(torch.cuda.current_stream(self.device))
        l = self.layer_index[layer_name]
        self._layer_store.layers(l, l + 1, stream=self._save_stream, wait_event=written)

    def end_layerwise_step(self) -> None:
        if self._layer_store is not None:
            ids = self._layer_store_ids
            self.store_futures[ids[0]] = (self._store_pool.submit(self._layer_store.finish), ids[1:])
            self._layer_store = None
        if self._layer_load is not None:
            # records stay pinned until the copies end; nothing to report
            self._layer_load_futures = [f for f in self._layer_load_futures if not f.done()]
            self._layer_load_futures.append(self._load_pool.submit(self._layer_load.finish))
            self._layer_load = None

    def lookup_agreed(self, keys_per_request: list[list[bytes]]) -> np.ndarray:
        """Per-request hit keys on this rank, min-reduced over the TP group."""
        hits = self.worker.lookup_batch(keys_per_request)
        return agree_min_hits(hits, self.tp_group)

    def _update_and_get_finished_store(self) -> set[str]:
        safe = self.finished_stores.intersection(self.previously_finished)
        self.finished_stores.difference_update(self.previously_finished)
        self.previously_finished.difference_update(safe)
        return safe

    def get_finished(self, finished_req_ids: set[str]) -> tuple[set[str] | None, set[str] | None]:
        finished_stores: set[str] = set()
        finished_loads: set[str] = set()
        for done, futs, what in ((finished_stores, self.store_futures, "store"),
                                 (finished_loads, self.load_futures, "retrieve")):
            for rid, (fut, others) in list(futs.items()):
                if not fut.done():
                    continue
                done.add(rid)
                done.update(others)
                out = fut.result() if fut.exception() is None else -1
                ret, per = out if isinstance(out, tuple) else (out, {})
                for r in [rid, *others]:
                    self.results[r] = per.get(r, ret)
                if ret != 0:   # reported but still finished, as the reference does (adaptor.py:243-265)
                    logger.error("Something went wrong when processing the %s request for request_id=%s, "
                                 "result=%s", what, rid, ret)
        for rid in finished_stores:
            self.store_futures.pop(rid, None)
        for rid in finished_loads:
            self.load_futures.pop(rid, None)
        self.finished_stores.update(finished_stores)
        ret_stores = set()
        for rid in finished_req_ids:
            if rid in self.finished_stores or rid in self.store_futures:
                self.previously_finished.add(rid)
            else:
                ret_stores.add(rid)
        ret_stores.update(self._update_and_get_finished_store())
        return ret_stores.intersection(finished_req_ids), finished_loads

    def wait_all(self, timeout: float | None = None) -> list[int]:
        """Block until every submitted store/load finished; their return codes."""
        out = []
        for d in (self.store_futures, self.load_futures):
            for fut, _ in d.values():
                r = fut.result(timeout=timeout)
                out.append(r[0] if isinstance(r, tuple) else r)
        return out
