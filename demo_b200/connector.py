"""vLLM KVConnectorBase_V1 implementation with the interface and scheduling
logic of CrossCache's python/crosscache_connector.py:1-688, backed by the
in-process adapters of demo_b200.adaptor.

Scheduler side (unchanged logic): a request tracker per request
(PREFETCHING -> WAITING_FOR_LOAD -> READY), chunk-granular store metadata for
fully scheduled, hashed, allocated blocks (GetStoreMetadata, :205-249) and
retrieve metadata for blocks [vllm_hit // bpc * bpc, cache_hit)
(GetRetrieveMetadata, :251-294).  Worker side: start_load_kv submits the
RETRIEVE ops, wait_for_save the STORE ops, get_finished reports them.

Configuration (kv_connector_extra_config): "cache.pool_size" bytes of pinned
host memory per (model, tp_size, tp_rank) entry (default 4 GiB, the
reference server's default, src/main.c:428).  With "cache.server.host"
(e.g. "tcp://localhost") and optionally "cache.server.port" (5555) set, as
the reference connector reads them (crosscache_connector.py:334-341), both
roles talk to a CrossCache server (python -m demo_b200.server) through the
adapters of demo_b200.remote instead of running the cache in-process.
"cache.layerwise": true (in-process only) turns on the layer pipeline the
reference leaves as no-ops (crosscache_connector.py:381-413): hits are
loaded inside the step that computes the request (load_async False), layer
by layer on a side stream, each attention layer waiting on the GPU for its
own layer (wait_for_layer_load); stores gather each layer as soon as the
forward has written it (save_kv_layer).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Literal, Optional, cast

import torch

from vllm.config import VllmConfig
from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1,
                                                               KVConnectorMetadata,
                                                               KVConnectorRole)
from vllm.logger import init_logger
from vllm.v1.core.sched.output import SchedulerOutput
from vllm.v1.utils import ConstantList

from .adaptor import LoadStoreOp, SchedulerAdapter, WorkerAdapter

logger = init_logger(__name__)

if TYPE_CHECKING:
    from vllm.forward_context import ForwardContext
    from vllm.v1.core.kv_cache_manager import KVCacheBlocks
    from vllm.v1.request import Request

# worker adapters registered in this process, by model name: the scheduler
# side answers lookups from the rank-0 worker's map (src/main.c:135-136)
_LOCAL_WORKERS: dict[str, WorkerAdapter] = {}


def reformat_block_ids(block_ids: tuple[list[int], ...] | None) -> list[int]:
    if block_ids is None:
        return []
    assert isinstance(block_ids, tuple), f"Expected block_ids to be a tuple of lists, but got {type(block_ids)}"
    if len(block_ids) > 1:
        raise RuntimeError("CrossCacheConnector only works without hybrid kv cache manager. "
                           "Please pass --disable-hybrid-kv-cache-manager when starting vllm")
    return block_ids[0]


def convert_block_hashes_to_bytes(block_hashes) -> list[bytes]:
    return cast(list[bytes], block_hashes)


class CacheRequestState(enum.Enum):
    PREFETCHING = enum.auto()
    WAITING_FOR_LOAD = enum.auto()
    READY = enum.auto()


@dataclass
class CacheRequestTracker:
    request_id: str
    all_token_ids: ConstantList[int]
    block_hashes: ConstantList
    allocated_block_ids: list[int] = field(default_factory=list)
    num_scheduled_tokens: int = 0
    num_stored_blocks: int = 0
    num_vllm_hit_blocks: int = 0
    num_cache_hit_blocks: int = 0
    state: CacheRequestState = CacheRequestState.PREFETCHING

    def __init__(self, request: "Request"):
        self.request_id = request.request_id
        self.all_token_ids = request.all_token_ids
        self.block_hashes = ConstantList(request.block_hashes)
        self.allocated_block_ids = []
        self.num_scheduled_tokens = 0
        self.num_stored_blocks = 0
        self.num_vllm_hit_blocks = 0
        self.num_cache_hit_blocks = 0
        self.state = CacheRequestState.PREFETCHING

    def needs_retrieve(self) -> bool:
        return self.num_cache_hit_blocks > self.num_vllm_hit_blocks and self.state != CacheRequestState.READY

    def is_ready_for_retrieving(self) -> bool:
        return self.state == CacheRequestState.WAITING_FOR_LOAD and self.needs_retrieve()

    def increase_num_scheduled_tokens(self, n: int) -> None:
        self.num_scheduled_tokens += n

    def increase_num_stored_blocks(self, n: int) -> None:
        self.num_stored_blocks += n

    def append_block_ids(self, new_block_ids: list[int]) -> None:
        self.allocated_block_ids.extend(new_block_ids)


@dataclass
class CacheRequestMetadata:
    request_id: str
    direction: Literal["STORE", "RETRIEVE"]
    op: LoadStoreOp

    @staticmethod
    def GetStoreMetadata(tracker: CacheRequestTracker, blocks_in_chunk: int,
                         vllm_block_size: int) -> "CacheRequestMetadata | None":
        min_available = min(len(tracker.block_hashes), len(tracker.allocated_block_ids),
                            tracker.num_scheduled_tokens // vllm_block_size)
        num_chunks = (min_available - tracker.num_stored_blocks) // blocks_in_chunk
        if num_chunks >= 1:
            start = tracker.num_stored_blocks
            end = start + num_chunks * blocks_in_chunk
            ret = CacheRequestMetadata(
                request_id=tracker.request_id, direction="STORE",
                op=LoadStoreOp(block_hashes=convert_block_hashes_to_bytes(tracker.block_hashes[start:end]),
                               block_ids=tracker.allocated_block_ids[start:end]))
            tracker.increase_num_stored_blocks(end - start)
            return ret
        return None

    @staticmethod
    def GetRetrieveMetadata(tracker: CacheRequestTracker, blocks_in_chunk: int) -> "CacheRequestMetadata | None":
        if not tracker.is_ready_for_retrieving():
            return None
        start = tracker.num_vllm_hit_blocks // blocks_in_chunk * blocks_in_chunk
        end = tracker.num_cache_hit_blocks
        assert end % blocks_in_chunk == 0
        assert len(tracker.block_hashes) >= end
        if end > start:
            return CacheRequestMetadata(
                request_id=tracker.request_id, direction="RETRIEVE",
                op=LoadStoreOp(block_hashes=convert_block_hashes_to_bytes(tracker.block_hashes[start:end]),
                               block_ids=tracker.allocated_block_ids[start:end]))
        return None


class CacheConnectorMetadata(KVConnectorMetadata):
    def __init__(self):
        super().__init__()
        self.requests: list[CacheRequestMetadata] = []

    def add_request_metadata(self, m: CacheRequestMetadata) -> None:
        self.requests.append(m)

    def __len__(self) -> int:
        return len(self.requests)


class CrossCacheConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config: "VllmConfig", role: KVConnectorRole, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        assert vllm_config.kv_transfer_config is not None
        pool_size = int(vllm_config.kv_transfer_config.get_from_extra_config("cache.pool_size", 4 << 30))
        model = vllm_config.model_config.model
        world_size = vllm_config.parallel_config.world_size
        rank = vllm_config.parallel_config.rank
        self.vllm_block_size = vllm_config.cache_config.block_size
        host = vllm_config.kv_transfer_config.get_from_extra_config("cache.server.host", None)
        self._remote = host is not None
        self._layerwise = bool(vllm_config.kv_transfer_config.get_from_extra_config("cache.layerwise", False))
        if self._layerwise and self._remote:
            raise ValueError("cache.layerwise needs the in-process cache (no cache.server.host)")
        self._step_stores: tuple[list[str], list[LoadStoreOp]] | None = None
        if self._remote:
            import zmq

            from .remote import RemoteSchedulerAdapter, RemoteWorkerAdapter
            port = vllm_config.kv_transfer_config.get_from_extra_config("cache.server.port", 5555)
            # the reference's host carries the scheme ("tcp://localhost"); a bare host means TCP
            url, ctx = f"{host if '://' in host else 'tcp://' + host}:{port}", zmq.Context.instance()
        if role == KVConnectorRole.SCHEDULER:
            if self._remote:
                self.scheduler_adapter = RemoteSchedulerAdapter(url, ctx, model, world_size, rank,
                                                                self.vllm_block_size)
            else:
                self.scheduler_adapter = SchedulerAdapter(model, world_size, rank, self.vllm_block_size)
            self.request_trackers: dict[str, CacheRequestTracker] = {}
        elif role == KVConnectorRole.WORKER:
            dev = torch.cuda.current_device()
            if self._remote:
                self.worker_adapter = RemoteWorkerAdapter(url, ctx, model, world_size, rank,
                                                          self.vllm_block_size, device=dev)
            else:
                self.worker_adapter = WorkerAdapter(model, world_size, rank, self.vllm_block_size,
                                                    pool_size=pool_size, device=dev)
        else:
            raise ValueError(f"Unknown KVConnectorRole: {role}")
        self._model = model

    # ---------------- worker side ----------------
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self.worker_adapter.register(kv_caches)
        if self.worker_adapter.worker_id == 0 and not self._remote:
            _LOCAL_WORKERS[self._model] = self.worker_adapter

    def wait_for_layer_load(self, layer_name: str) -> None:
        if self._layerwise:
            self.worker_adapter.wait_layer(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kwargs: Any) -> None:
        if not self._layerwise:
            return
        if self._step_stores is None:
            metadata = self._get_connector_metadata()
            assert isinstance(metadata, CacheConnectorMetadata)
            ids, ops = [], []
            for m in metadata.requests:
                if m.direction == "STORE":
                    ids.append(m.request_id)
                    ops.append(m.op)
            self._step_stores = (ids, ops)
        ids, ops = self._step_stores
        if ids:
            self.worker_adapter.save_layer(layer_name, ids, ops)

    def start_load_kv(self, forward_context: "ForwardContext", **kwargs: Any) -> None:
        metadata = self._get_connector_metadata()
        assert isinstance(metadata, CacheConnectorMetadata)
        ids, ops = [], []
        for m in metadata.requests:
            if m.direction == "RETRIEVE":
                ids.append(m.request_id)
                ops.append(m.op)
        if ids:
            if self._layerwise:
                self.worker_adapter.begin_layerwise_load(ids, ops)
            else:
                self.worker_adapter.load_requests(ids, ops)

    def wait_for_save(self):
        if self._layerwise:
            layered = self._step_stores is not None
            self._step_stores = None
            self.worker_adapter.end_layerwise_step()
            if layered:
                return
            # no save_kv_layer call this step: store whole records instead
        metadata = self._get_connector_metadata()
        assert isinstance(metadata, CacheConnectorMetadata)
        ids, ops = [], []
        for m in metadata.requests:
            if m.direction == "STORE":
                ids.append(m.request_id)
                ops.append(m.op)
        if ids:
            self.worker_adapter.store_requests(ids, ops)

    def get_finished(self, finished_req_ids: set[str]) -> tuple[set[str] | None, set[str] | None]:
        return self.worker_adapter.get_finished(finished_req_ids)

    def get_block_ids_with_load_errors(self) -> set[int]:
        """Blocks whose load failed (a record evicted or unreadable between
        lookup and load): vLLM recomputes them.  The reference logs the
        failure and lets the request run on whatever the blocks held."""
        take = getattr(self.worker_adapter, "take_failed_load_blocks", None) if hasattr(
            self, "worker_adapter") else None
        return take() if take is not None else set()

    def shutdown(self):
        if hasattr(self, "worker_adapter"):
            if not self._remote:
                _LOCAL_WORKERS.pop(self._model, None)
            self.worker_adapter.unregister()
        if self._remote and hasattr(self, "scheduler_adapter"):
            self.scheduler_adapter.close()
        return None

    # ---------------- scheduler side ----------------
    def _lookup_worker(self):
        wa = _LOCAL_WORKERS.get(self._model)
        return wa.worker if wa is not None else None

    def get_num_new_matched_tokens(self, request: "Request", num_computed_tokens: int) -> tuple[int | None, bool]:
        tracker = self._get_or_create_request_tracker(request)
        if not self._remote and self.scheduler_adapter._worker is None:
            w = self._lookup_worker()
            if w is not None:
                self.scheduler_adapter.bind_worker(w)
        self.scheduler_adapter.try_lookup(request.request_id, convert_block_hashes_to_bytes(request.block_hashes))
        ret = self.scheduler_adapter.check_lookup_result(request.request_id)
        if ret is None:
            return None, True
        if ret == 0:
            return 0, False
        assert ret % (self.scheduler_adapter.num_blocks_per_chunk() * self.vllm_block_size) == 0
        num_vllm_blocks = num_computed_tokens // self.vllm_block_size
        num_cache_blocks = ret // self.vllm_block_size
        tracker.increase_num_stored_blocks(num_cache_blocks)
        tracker.num_vllm_hit_blocks = num_vllm_blocks
        tracker.num_cache_hit_blocks = num_cache_blocks
        need_to_load = max(0, ret - num_computed_tokens)
        if not self._layerwise:
            return need_to_load, need_to_load > 0
        # layer-wise: loaded inside the step that computes the request.  That
        # step must compute at least one token (vLLM trims a full hit itself
        # only for asynchronous loads), so a hit covering the whole prompt
        # leaves its last token to the forward; the load still moves whole
        # records, and the forward rewrites that token's slot with its own
        # K/V.
        if num_computed_tokens + need_to_load >= request.num_tokens:
            need_to_load = max(0, request.num_tokens - 1 - num_computed_tokens)
        return need_to_load, False

    def update_state_after_alloc(self, request: "Request", blocks: "KVCacheBlocks", num_external_tokens: int):
        tracker = self._get_request_tracker(request.request_id)
        tracker.append_block_ids(reformat_block_ids(blocks.get_block_ids()))
        condition = tracker.needs_retrieve()
        if tracker.state == CacheRequestState.PREFETCHING:
            tracker.state = CacheRequestState.WAITING_FOR_LOAD if condition else CacheRequestState.READY
            self.scheduler_adapter.cleanup_lookup_result(request.request_id)

    def build_connector_meta(self, scheduler_output: SchedulerOutput) -> KVConnectorMetadata:
        metadata = CacheConnectorMetadata()
        self._process_retrieve_requests(metadata)
        self._process_new_requests(scheduler_output, metadata)
        self._process_cached_requests(scheduler_output, metadata)
        return metadata

    def request_finished(self, request: "Request", block_ids: list[int]) -> tuple[bool, dict[str, Any] | None]:
        self.request_trackers.pop(request.request_id, None)
        self.scheduler_adapter.cleanup_lookup_result(request.request_id)
        return True, None

    def _process_retrieve_requests(self, metadata: CacheConnectorMetadata) -> None:
        bpc = self.scheduler_adapter.num_blocks_per_chunk()
        for t in self.request_trackers.values():
            if t.state != CacheRequestState.WAITING_FOR_LOAD:
                continue
            m = CacheRequestMetadata.GetRetrieveMetadata(t, bpc)
            if m is not None:
                metadata.add_request_metadata(m)
            t.state = CacheRequestState.READY

    def _process_new_requests(self, scheduler_output: SchedulerOutput, metadata: CacheConnectorMetadata) -> None:
        bpc = self.scheduler_adapter.num_blocks_per_chunk()
        for new in scheduler_output.scheduled_new_reqs:
            t = self._get_request_tracker(new.req_id)
            t.increase_num_scheduled_tokens(scheduler_output.num_scheduled_tokens[new.req_id])
            m = CacheRequestMetadata.GetStoreMetadata(t, bpc, self.vllm_block_size)
            if m is not None:
                metadata.add_request_metadata(m)

    def _process_cached_requests(self, scheduler_output: SchedulerOutput, metadata: CacheConnectorMetadata) -> None:
        bpc = self.scheduler_adapter.num_blocks_per_chunk()
        cached = scheduler_output.scheduled_cached_reqs
        for idx, rid in enumerate(cached.req_ids):
            t = self._get_request_tracker(rid)
            t.append_block_ids(reformat_block_ids(cached.new_block_ids[idx]))
            # the reference adds num_computed_tokens here (crosscache_connector.py:653)
            t.increase_num_scheduled_tokens(cached.num_computed_tokens[idx])
            m = CacheRequestMetadata.GetStoreMetadata(t, bpc, self.vllm_block_size)
            if m is not None:
                metadata.add_request_metadata(m)

    def _get_request_tracker(self, request_id: str) -> CacheRequestTracker:
        assert request_id in self.request_trackers, f"Request tracker for request_id {request_id} not found. "
        return self.request_trackers[request_id]

    def _get_or_create_request_tracker(self, request: "Request") -> CacheRequestTracker:
        if request.request_id not in self.request_trackers:
            self.request_trackers[request.request_id] = CacheRequestTracker(request)
        return self.request_trackers[request.request_id]
