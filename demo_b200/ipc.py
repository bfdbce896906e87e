"""CUDA IPC keys for paged-KV layer tensors.

CUDA counterpart of CrossCache's python/ipckey_utils.cpp:19-33
(ipckey_from_tensor -> aclrtIpcMemGetExportKey, 64 bytes).  PyTorch
sub-allocates tensors inside larger cudaMalloc blocks, and a
cudaIpcMemHandle_t names the whole block, so a key here is 72 bytes: the
64-byte handle followed by the little-endian uint64 byte offset of the
tensor's first element inside that block.  open_ipc_keys (include/device.h)
accepts such keys with per_len 72.
"""
from __future__ import annotations

import torch

IPC_HANDLE_BYTES = 64
KEY_BYTES = IPC_HANDLE_BYTES + 8


def ipckey_from_ptr(ptr: int) -> bytes:
    """72-byte key of a device address (include/device.h ipc_export_key):
    handle of the enclosing cudaMalloc block + byte offset of `ptr`."""
    import ctypes as C

    from ._lib import lib

    buf = (C.c_uint8 * KEY_BYTES)()
    ret = lib.ipc_export_key(C.c_void_p(ptr), buf)
    if ret:
        raise RuntimeError(f"ipc_export_key failed: {ret}")
    return bytes(buf)


def ipckey_from_tensor(t: torch.Tensor) -> bytes:
    """72-byte key of the tensor's first element (ipckey_from_ptr)."""
    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return ipckey_from_ptr(t.data_ptr())


def layer_keys(kv_caches) -> tuple[bytes, bytes | None]:
    """Concatenated K keys and V keys (None for a K-only cache) of per-layer
    vLLM KV tensors (the forms demo_b200.cache.layout_from_kv_tensors
    takes): the key of each layer's K plane and V plane base -- the
    k_raw_ptrs / v_raw_ptrs of a worker_context registered with per_len 72."""
    from . import cache as cc

    layers = list(kv_caches)
    if any(not t.is_cuda for t in layers):
        raise ValueError("KV tensors must be on a CUDA device")
    _, kp, vp = cc.layout_from_kv_tensors(layers)
    ks = b"".join(ipckey_from_ptr(p) for p in kp)
    return ks, (b"".join(ipckey_from_ptr(p) for p in vp) if vp is not None else None)
