"""In-process Python front end of the cache-manager C API (include/cache.h).

CrossCache's vLLM worker hands its KV tensors to a separate C server over
ZeroMQ + Ascend IPC keys (python/adaptor.py:149-228, src/main.c:244-348).
This module drives the same C API in the worker's own process: the paged KV
tensors are registered by raw device pointer (per_len 8), and keys / block
ids go straight to cache_store / cache_load / cache_lookup.  PyTorch is used
only to read tensor pointers and shapes.
"""
from __future__ import annotations

import ctypes as C
import errno
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from ._lib import (CACHE_BACKEND_CUDA, CACHE_BACKEND_MEM, CacheStats, ModelInfo, WorkerContext,
                   lib)

KEY_LEN = 32
_chunk_size = 256          # tokens per record of the running cache (init)


class CacheError(RuntimeError):
    def __init__(self, what: str, ret: int):
        name = errno.errorcode.get(-ret, str(ret)) if ret < 0 else str(ret)
        super().__init__(f"{what} failed: {ret} ({name})")
        self.ret = ret


def init(chunk_size: int = 256, pool_size: int = 4 << 30, root_dir: str | None = None,
         backend: int = CACHE_BACKEND_CUDA) -> None:
    """cache_init (CrossCache cache.c:759-787) with an explicit backend."""
    global _chunk_size
    ret = lib.cache_init_backend(chunk_size, pool_size, root_dir.encode() if root_dir else None, backend)
    if ret:
        raise CacheError("cache_init", ret)
    _chunk_size = chunk_size


def exit() -> None:  # noqa: A001 - mirrors cache_exit
    lib.cache_exit()


def _keys_buffer(keys: Sequence[bytes]) -> bytes:
    for k in keys:
        if len(k) != KEY_LEN:
            raise ValueError(f"keys must be {KEY_LEN} bytes (got {len(k)})")
    return b"".join(keys)


@dataclass
class KVLayout:
    num_layers: int
    num_blocks: int
    block_size: int
    hidden_dim_size: int     # heads * head_dim of this rank
    element_size: int
    kv: int                  # 2 = K and V, 1 = K only (MLA)
    # paged geometry of the planes (cache_register_paged, include/cache.h):
    # 0 / 0 = dense token-major, the reference's FlashAttention layout
    block_stride: int = 0    # bytes from one block of a plane to the next
    head_bytes: int = 0      # > 0: head-major blocks [heads][block_size][head_bytes]

    @property
    def unit(self) -> int:
        return self.hidden_dim_size * self.element_size

    @property
    def per_token_size(self) -> int:
        return self.kv * self.num_layers * self.unit


class Worker:
    """One registered worker: a (model, world_size, rank) entry of the cache.

    `k_ptrs` / `v_ptrs` are per-layer base addresses of the K and V planes
    (device pointers for the CUDA backend, host pointers for the MEM backend).
    """

    def __init__(self, model_name: str, layout: KVLayout, k_ptrs: Sequence[int],
                 v_ptrs: Sequence[int] | None, node_id: int = 0, world_size: int = 1,
                 rank: int = 0):
        if len(k_ptrs) != layout.num_layers or (v_ptrs is not None and len(v_ptrs) != layout.num_layers):
            raise ValueError("one pointer per layer")
        if (v_ptrs is None) != (layout.kv == 1):
            raise ValueError("layout.kv must be 1 exactly when v_ptrs is None")
        self.layout = layout
        self._name = model_name.encode()
        self._k = np.asarray(k_ptrs, dtype=np.uint64)
        self._v = np.asarray(v_ptrs, dtype=np.uint64) if v_ptrs is not None else None
        self.ctx = WorkerContext()
        self.ctx.model = ModelInfo(self._name, layout.element_size, layout.num_layers, layout.hidden_dim_size)
        self.ctx.node_id = node_id
        self.ctx.world_size = world_size
        self.ctx.rank_id = rank
        self.ctx.per_token_size = layout.per_token_size
        self.ctx.num_blocks = layout.num_blocks
        self.ctx.block_size = layout.block_size
        self.ctx.per_len = 8
        self.ctx.k_raw_ptrs = self._k.ctypes.data
        self.ctx.v_raw_ptrs = self._v.ctypes.data if self._v is not None else None
        self.registered = False

    @classmethod
    def from_keys(cls, model_name: str, layout: KVLayout, k_keys: bytes, v_keys: bytes | None,
                  per_len: int, node_id: int = 0, world_size: int = 1, rank: int = 0) -> "Worker":
        """A worker registered from per-layer keys of `per_len` bytes each
        (8: raw pointers of this process, 64: CUDA IPC handles, 72: handle +
        offset) -- what the server receives in a REGISTER message."""
        if len(k_keys) != layout.num_layers * per_len or (
                v_keys is not None and len(v_keys) != layout.num_layers * per_len):
            raise ValueError("one key of per_len bytes per layer")
        w = cls(model_name, layout, [0] * layout.num_layers,
                [0] * layout.num_layers if v_keys is not None else None, node_id, world_size, rank)
        w._kbuf = C.create_string_buffer(bytes(k_keys), len(k_keys))
        w._vbuf = C.create_string_buffer(bytes(v_keys), len(v_keys)) if v_keys is not None else None
        w.ctx.per_len = per_len
        w.ctx.k_raw_ptrs = C.cast(w._kbuf, C.c_void_p)
        w.ctx.v_raw_ptrs = C.cast(w._vbuf, C.c_void_p) if w._vbuf is not None else None
        return w

    # -- reference API ------------------------------------------------------
    def register(self) -> None:
        lay = self.layout
        if lay.block_stride or lay.head_bytes:
            ret = lib.cache_register_paged(C.byref(self.ctx), lay.block_stride, lay.head_bytes)
        else:
            ret = lib.cache_register(C.byref(self.ctx))
        if ret:
            raise CacheError("cache_register", ret)
        self.registered = True

    def unregister(self) -> None:
        if self.registered:
            lib.cache_unregister(C.byref(self.ctx))
            self.registered = False

    def store(self, keys: Sequence[bytes], block_ids: Sequence[int]) -> int:
        """cache_store: returns 0 or a negative errno (reference semantics)."""
        kb = _keys_buffer(keys)
        b = np.ascontiguousarray(np.asarray(block_ids, dtype=np.uint64))
        return lib.cache_store(C.byref(self.ctx), kb, KEY_LEN, b.ctypes.data, len(b))

    def load(self, keys: Sequence[bytes], block_ids: Sequence[int]) -> int:
        kb = _keys_buffer(keys)
        b = np.ascontiguousarray(np.asarray(block_ids, dtype=np.uint64))
        return lib.cache_load(C.byref(self.ctx), kb, KEY_LEN, b.ctypes.data, len(b))

    def lookup(self, keys: Sequence[bytes]) -> int:
        """cache_lookup: byte offset of the first miss (hit keys * 32)."""
        kb = _keys_buffer(keys)
        return lib.cache_lookup(C.byref(self.ctx), kb, len(keys), KEY_LEN)

    # -- additions ----------------------------------------------------------
    def lookup_batch(self, keys_per_request: Sequence[Sequence[bytes]]) -> np.ndarray:
        """cache_lookup_batch: leading hit keys per request."""
        nums = np.array([len(k) for k in keys_per_request], dtype=np.uint32)
        kb = b"".join(_keys_buffer(k) for k in keys_per_request)
        out = np.zeros(len(nums), dtype=np.uint32)
        ret = lib.cache_lookup_batch(C.byref(self.ctx), kb, nums.ctypes.data, len(nums), KEY_LEN,
                                     out.ctypes.data)
        if ret and ret != -errno.ENOENT:
            raise CacheError("cache_lookup_batch", ret)
        return out

    def store_batch(self, keys_per_request: Sequence[Sequence[bytes]],
                    block_ids_per_request: Sequence[Sequence[int]]) -> tuple[int, np.ndarray]:
        """cache_store_batch: (overall result, per-request results)"""
        return self._batch(lib.cache_store_batch, keys_per_request, block_ids_per_request)

    def load_batch(self, keys_per_request: Sequence[Sequence[bytes]],
                   block_ids_per_request: Sequence[Sequence[int]]) -> tuple[int, np.ndarray]:
        """cache_load_batch: (overall result, per-request results)"""
        return self._batch(lib.cache_load_batch, keys_per_request, block_ids_per_request)

    def _batch(self, fn, keys_per_request, block_ids_per_request):
        nums = np.array([len(k) for k in keys_per_request], dtype=np.uint32)
        bpc = _chunk_size // self.layout.block_size
        if len(keys_per_request) != len(block_ids_per_request) or any(
                len(bl) != len(k) * bpc for k, bl in zip(keys_per_request, block_ids_per_request)):
            raise ValueError(f"each request needs {bpc} block ids per key")
        kb = b"".join(_keys_buffer(k) for k in keys_per_request)
        b = np.ascontiguousarray(np.concatenate(
            [np.asarray(x, dtype=np.uint64) for x in block_ids_per_request]) if len(nums) else
            np.zeros(0, np.uint64))
        st = np.zeros(len(nums), dtype=np.int32)
        ret = fn(C.byref(self.ctx), kb, KEY_LEN, nums.ctypes.data, len(nums), b.ctypes.data, st.ctypes.data)
        return ret, st

    def stats(self) -> dict:
        s = CacheStats()
        ret = lib.cache_get_stats(C.byref(self.ctx), C.byref(s))
        if ret:
            raise CacheError("cache_get_stats", ret)
        return s.as_dict()

    def clear(self) -> None:
        ret = lib.cache_clear(C.byref(self.ctx))
        if ret:
            raise CacheError("cache_clear", ret)

    def load_async(self, keys: Sequence[bytes], block_ids: Sequence[int]) -> "AsyncTransfer":
        """cache_load_async: pins the cached records of `keys` (the others are
        skipped; .missing says whether any was); move them with .layers()."""
        return self._async(lib.cache_load_async, keys, block_ids)

    def store_async(self, keys: Sequence[bytes], block_ids: Sequence[int]) -> "AsyncTransfer":
        """cache_store_async: reserves records for the new keys; move them
        with .layers() (every layer, or .finish() drops them)."""
        return self._async(lib.cache_store_async, keys, block_ids)

    def _async(self, fn, keys, block_ids) -> "AsyncTransfer":
        kb = _keys_buffer(keys)
        b = np.ascontiguousarray(np.asarray(block_ids, dtype=np.uint64))
        h = C.c_void_p()
        ret = fn(C.byref(self.ctx), kb, KEY_LEN, b.ctypes.data, len(b), C.byref(h))
        if ret and ret != -errno.ENOENT:
            raise CacheError(fn.__name__, ret)
        return AsyncTransfer(h, missing=ret == -errno.ENOENT)

    def flush(self) -> None:
        """cache_flush: wait for the disk writes of every stored record."""
        ret = lib.cache_flush(C.byref(self.ctx))
        if ret:
            raise CacheError("cache_flush", ret)


def _handle(x) -> int | None:
    """cudaStream_t / cudaEvent_t of a torch stream or event, an int, or None"""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    for attr in ("cuda_stream", "cuda_event"):
        if hasattr(x, attr):
            return getattr(x, attr)
    raise TypeError(f"not a CUDA stream or event: {x!r}")


class AsyncTransfer:
    """Handle of cache_load_async / cache_store_async."""

    def __init__(self, handle: C.c_void_p, missing: bool = False):
        self._h = handle
        self.missing = missing

    @property
    def records(self) -> int:
        return lib.cache_async_records(self._h)

    def layers(self, begin: int, end: int, stream=None, wait_event=None) -> None:
        """enqueue layers [begin, end) on `stream` after `wait_event`"""
        ret = lib.cache_async_layers(self._h, begin, end, _handle(stream), _handle(wait_event))
        if ret:
            raise CacheError("cache_async_layers", ret)

    def stream_wait(self, layer: int, stream=None) -> None:
        """make `stream` wait on the GPU for the copy covering `layer`"""
        ret = lib.cache_async_stream_wait(self._h, layer, _handle(stream))
        if ret:
            raise CacheError("cache_async_stream_wait", ret)

    def query(self) -> bool:
        ret = lib.cache_async_query(self._h)
        if ret < 0:
            raise CacheError("cache_async_query", ret)
        return ret == 1

    def finish(self) -> int:
        """cache_async_finish: 0 or a negative errno; the handle is released"""
        if self._h is None:
            return 0
        h, self._h = self._h, None
        return lib.cache_async_finish(h)


def _plane_geometry(nb: int, bs: int, h: int, d: int, strides, esz: int) -> tuple[int, int]:
    """(block_stride, head_bytes) of a plane indexed [block][token][head][dim]
    with element strides `strides`; ValueError for a geometry the kernels
    cannot address"""
    sb, st, sh, sd = strides
    if d > 1 and sd != 1:
        raise ValueError("head_dim must be the innermost, contiguous dimension")
    unit = h * d
    if (h == 1 or sh == d) and st == unit:               # token-major block
        head_bytes = 0
    elif st == d and sh == bs * d:                        # head-major block (HND)
        head_bytes = d * esz
    else:
        raise ValueError(f"unsupported KV block strides {tuple(strides)}")
    if nb > 1 and sb < bs * unit:
        raise ValueError("KV blocks overlap")
    block_stride = sb * esz if nb > 1 else bs * unit * esz
    if block_stride == bs * unit * esz and not head_bytes:
        block_stride = 0                                  # dense: the reference layout
    return block_stride, head_bytes


def layout_from_kv_tensors(kv_caches, kv_layout: str | None = None
                           ) -> tuple[KVLayout, list[int], list[int] | None]:
    """Layout and per-layer K/V plane pointers of vLLM paged caches.

    kv_caches: iterable of per-layer tensors, all of one shape, strides and
    dtype, each either
      [2, num_blocks, block_size, heads, head_dim]  FlashAttention: K plane
          then V plane (the reference's layout, src python connector)
      [num_blocks, 2, block_size, heads, head_dim]  FlashInfer: K and V of a
          block side by side; on sm_100 vLLM stores the block head-major
          (the tensor is a permuted view of [num_blocks, 2, heads,
          block_size, head_dim])
      [num_blocks, block_size, width]               K-only MLA latent cache
    The two 5-d forms are told apart by which leading dimension is 2;
    `kv_layout` ("flash_attn" / "flashinfer") settles a cache of 2 blocks.
    Strided or head-major blocks come back as a non-zero
    KVLayout.block_stride / head_bytes (cache_register_paged).
    """
    layers = list(kv_caches)
    if not layers:
        raise ValueError("no KV layer tensors")
    t0 = layers[0]
    esz = t0.element_size()
    for t in layers:
        if t.shape != t0.shape or t.stride() != t0.stride() or t.dtype != t0.dtype:
            raise ValueError("KV layer tensors must share one shape, strides and dtype")
    if t0.dim() == 5:
        if kv_layout is None:
            if t0.shape[0] == 2 and t0.shape[1] != 2:
                kv_layout = "flash_attn"
            elif t0.shape[1] == 2 and t0.shape[0] != 2:
                kv_layout = "flashinfer"
            else:
                raise ValueError(f"ambiguous KV tensor shape {tuple(t0.shape)}: pass kv_layout")
        if kv_layout == "flash_attn":
            _, nb, bs, h, d = t0.shape
            skv, sb, st, sh, sd = t0.stride()
        elif kv_layout == "flashinfer":
            nb, _, bs, h, d = t0.shape
            sb, skv, st, sh, sd = t0.stride()
        else:
            raise ValueError(f"unknown kv_layout {kv_layout!r}")
        kv = 2
        hidden = h * d
        block_stride, head_bytes = _plane_geometry(nb, bs, h, d, (sb, st, sh, sd), esz)
        k = [t.data_ptr() for t in layers]
        v = [t.data_ptr() + skv * esz for t in layers]
    elif t0.dim() == 3:
        nb, bs, hidden = t0.shape
        sb, st, sd = t0.stride()
        kv = 1
        block_stride, head_bytes = _plane_geometry(nb, bs, 1, hidden, (sb, st, hidden, sd), esz)
        k, v = [t.data_ptr() for t in layers], None
    else:
        raise ValueError(f"unsupported KV tensor shape {tuple(t0.shape)}")
    lay = KVLayout(num_layers=len(layers), num_blocks=int(nb), block_size=int(bs),
                   hidden_dim_size=int(hidden), element_size=esz, kv=kv,
                   block_stride=int(block_stride), head_bytes=int(head_bytes))
    return lay, k, v


__all__ = ["init", "exit", "Worker", "KVLayout", "layout_from_kv_tensors", "CacheError",
           "CACHE_BACKEND_CUDA", "CACHE_BACKEND_MEM", "KEY_LEN"]
