"""ctypes bindings of libcrosscache.so (the C ABI declared in include/*.h).

Importing this module loads the in-tree library and raises if it is missing:
there is no Python or CPU stand-in for the CUDA path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcrosscache.so"

CACHE_BACKEND_CUDA = 0
CACHE_BACKEND_MEM = 1

KVCOPY_ERR_SLOT_RANGE = 0x1
KVCOPY_ERR_NULL_LAYER = 0x2
KVCOPY_ERR_TIMEOUT = 0x4
KVCOPY_ERR_ALIGN = 0x8
KVCOPY_FLAG_BULK = 0x1
KVCOPY_FLAG_TEST_STALL = 0x100
KVCOPY_PATH_REGISTER, KVCOPY_PATH_BULK, KVCOPY_PATH_BULK_HND = 1, 2, 3
KVHASH_MAX_BLOCK_SIZE = 8192
KVHASH_ALGOS = {"sha256": 0, "sha256_cbor": 1}


class ModelInfo(C.Structure):
    _fields_ = [
        ("model_name", C.c_char_p),
        ("element_size", C.c_uint8),
        ("num_layers", C.c_uint8),
        ("hidden_dim_size", C.c_uint32),
    ]


class WorkerContext(C.Structure):
    """struct worker_context (include/inner.h; CrossCache include/inner_h/inner.h:6-30)."""

    _fields_ = [
        ("model", ModelInfo),
        ("node_id", C.c_uint8),
        ("world_size", C.c_uint8),
        ("rank_id", C.c_uint8),
        ("per_token_size", C.c_uint32),
        ("num_blocks", C.c_uint32),
        ("block_size", C.c_uint32),
        ("per_len", C.c_uint16),
        ("k_raw_ptrs", C.c_void_p),
        ("v_raw_ptrs", C.c_void_p),
        ("k_ptrs", C.c_void_p),
        ("v_ptrs", C.c_void_p),
    ]


class TransferParams(C.Structure):
    """struct transfer_params (include/device.h; CrossCache device.h:13-28)."""

    _fields_ = [
        ("caches", C.c_void_p),
        ("caches_h", C.c_void_p),
        ("keys_ptrs", C.c_void_p),
        ("value_ptrs", C.c_void_p),
        ("page_buffer_size", C.c_uint64),
        ("slot_mapping", C.c_void_p),
        ("devid", C.c_uint8),
        ("caches_element_size", C.c_uint8),
        ("num_layers", C.c_uint16),
        ("num_tokens", C.c_uint16),
        ("hidden_dim_size", C.c_uint32),
        ("direction", C.c_bool),
    ]


class TransferBatch(C.Structure):
    """struct transfer_batch (include/device.h, new)."""

    _fields_ = [
        ("keys_ptrs", C.c_void_p),
        ("value_ptrs", C.c_void_p),
        ("page_buffer_size", C.c_uint64),
        ("records", C.POINTER(C.c_void_p)),
        ("block_ids", C.POINTER(C.c_uint64)),
        ("num_records", C.c_uint32),
        ("block_size", C.c_uint32),
        ("hidden_dim_size", C.c_uint32),
        ("num_layers", C.c_uint16),
        ("num_tokens", C.c_uint16),
        ("devid", C.c_uint8),
        ("caches_element_size", C.c_uint8),
        ("record_on_device", C.c_uint8),
        ("direction", C.c_bool),
        ("block_stride", C.c_uint64),
        ("head_bytes", C.c_uint32),
    ]


class KvCopyDesc(C.Structure):
    """struct kv_copy_desc (include/kvcopy.h)."""

    _fields_ = [
        ("layer_k", C.c_void_p),
        ("layer_v", C.c_void_p),
        ("records", C.c_void_p),
        ("slots", C.c_void_p),
        ("block_ids", C.c_void_p),
        ("error", C.c_void_p),
        ("page_buffer_size", C.c_uint64),
        ("unit_bytes", C.c_uint32),
        ("num_tokens", C.c_uint32),
        ("block_size", C.c_uint32),
        ("num_layers", C.c_uint32),
        ("num_records", C.c_uint32),
        ("direction", C.c_int32),
        ("flags", C.c_uint32),
        ("layer_begin", C.c_uint32),
        ("record_layers", C.c_uint32),
        ("max_ctas", C.c_uint32),
        ("block_stride", C.c_uint64),
        ("head_bytes", C.c_uint32),
    ]


class CacheStats(C.Structure):
    """struct cache_stats (include/cache.h, new)."""

    _fields_ = [(n, C.c_uint64) for n in (
        "records_total", "records_used", "lookups", "lookup_hits", "stored",
        "store_dedup", "loaded", "load_misses", "evictions", "bytes_saved", "bytes_loaded",
        "disk_writes", "disk_write_skips", "disk_write_errors", "disk_reads", "disk_read_errors",
        "disk_lookup_hits", "bytes_written_disk", "bytes_read_disk")]

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


# exported symbol -> (restype, argtypes); every entry point of include/*.h
SIGNATURES: dict[str, tuple] = {
    # include/cache.h
    "cache_init": (C.c_int, [C.c_uint32, C.c_uint64, C.c_char_p]),
    "cache_init_backend": (C.c_int, [C.c_uint32, C.c_uint64, C.c_char_p, C.c_int]),
    "cache_exit": (None, []),
    "cache_register": (C.c_int, [C.POINTER(WorkerContext)]),
    "cache_register_paged": (C.c_int, [C.POINTER(WorkerContext), C.c_uint64, C.c_uint32]),
    "cache_unregister": (None, [C.POINTER(WorkerContext)]),
    "cache_lookup": (C.c_int, [C.POINTER(WorkerContext), C.c_void_p, C.c_uint32, C.c_uint32]),
    "cache_store": (C.c_int, [C.POINTER(WorkerContext), C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "cache_load": (C.c_int, [C.POINTER(WorkerContext), C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "cache_lookup_batch": (C.c_int, [C.POINTER(WorkerContext), C.c_void_p, C.c_void_p, C.c_uint32,
                                     C.c_uint32, C.c_void_p]),
    "cache_get_stats": (C.c_int, [C.POINTER(WorkerContext), C.POINTER(CacheStats)]),
    "cache_clear": (C.c_int, [C.POINTER(WorkerContext)]),
    "cache_flush": (C.c_int, [C.POINTER(WorkerContext)]),
    "cache_store_batch": (C.c_int, [C.POINTER(WorkerContext), C.c_char_p, C.c_uint32, C.c_void_p, C.c_uint32,
                                    C.c_void_p, C.c_void_p]),
    "cache_load_batch": (C.c_int, [C.POINTER(WorkerContext), C.c_char_p, C.c_uint32, C.c_void_p, C.c_uint32,
                                   C.c_void_p, C.c_void_p]),
    "cache_load_async": (C.c_int, [C.POINTER(WorkerContext), C.c_char_p, C.c_uint32, C.c_void_p, C.c_uint32,
                                   C.POINTER(C.c_void_p)]),
    "cache_store_async": (C.c_int, [C.POINTER(WorkerContext), C.c_char_p, C.c_uint32, C.c_void_p, C.c_uint32,
                                    C.POINTER(C.c_void_p)]),
    "cache_async_layers": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]),
    "cache_async_stream_wait": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p]),
    "cache_async_query": (C.c_int, [C.c_void_p]),
    "cache_async_finish": (C.c_int, [C.c_void_p]),
    "cache_async_records": (C.c_uint32, [C.c_void_p]),
    # include/device.h
    "cuda_adaptor_create": (C.c_void_p, []),
    "cuda_adaptor_destroy": (None, [C.c_void_p]),
    "mem_adaptor_create": (C.c_void_p, []),
    "mem_adaptor_destroy": (None, [C.c_void_p]),
    "alloc_pinned_ptr": (C.c_void_p, [C.c_void_p, C.c_uint8, C.c_uint64, C.c_uint, C.POINTER(C.c_void_p)]),
    "free_pinned_ptr": (None, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "wrapper_ptr": (C.c_void_p, [C.c_void_p, C.c_uint8, C.c_void_p, C.c_uint64]),
    "unwrapper_ptr": (None, [C.c_void_p, C.c_void_p]),
    "open_ipc_keys": (C.c_void_p, [C.c_void_p, C.c_uint8, C.c_uint16, C.c_uint16, C.c_void_p]),
    "close_ipc_keys": (None, [C.c_void_p, C.c_void_p]),
    "transfer_kvcache": (C.c_int, [C.c_void_p, C.POINTER(TransferParams)]),
    "transfer_kvcache_batch": (C.c_int, [C.c_void_p, C.POINTER(TransferBatch)]),
    "transfer_async_begin": (C.c_void_p, [C.c_void_p, C.POINTER(TransferBatch), C.POINTER(C.c_int)]),
    "transfer_async_layers": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]),
    "transfer_async_stream_wait": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]),
    "transfer_async_query": (C.c_int, [C.c_void_p, C.c_void_p]),
    "transfer_async_end": (C.c_int, [C.c_void_p, C.c_void_p]),
    "reset_device": (None, [C.c_void_p, C.c_uint8]),
    "crosscache_kernel_launches": (C.c_uint64, []),
    "ipc_export_key": (C.c_int, [C.c_void_p, C.c_void_p]),
    # include/kvcopy.h
    "kv_copy_launch": (C.c_int, [C.POINTER(KvCopyDesc), C.c_void_p]),
    "kv_copy_payload_bytes": (C.c_uint64, [C.POINTER(KvCopyDesc)]),
    "kv_copy_path": (C.c_int, [C.POINTER(KvCopyDesc)]),
    "kv_copy_noalloc": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                  C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int32,
                                  C.c_uint32, C.c_void_p]),
    # include/kvhash.h
    "kv_block_hash_launch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kv_block_hash_host": (C.c_int64, [C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                       C.c_void_p, C.c_void_p]),
    "kv_block_hash_launch_algo": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_int,
                                            C.c_void_p]),
    "kv_block_hash_host_algo": (C.c_int64, [C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                            C.c_void_p, C.c_void_p, C.c_int]),
    "kv_block_hash_launch_ext": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_int, C.c_void_p]),
    "kv_block_hash_host_ext": (C.c_int64, [C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
}


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built; run `python -m demo_b200.build` (nvcc for sm_100a). "
            "There is no fallback implementation.")
    lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
