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


def ipckey_from_tensor(t: torch.Tensor) -> bytes:
    """72-byte key of the tensor's first element (include/device.h
    ipc_export_key): handle of the enclosing cudaMalloc block + byte offset."""
    import ctypes as C

    from ._lib import lib

    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    buf = (C.c_uint8 * KEY_BYTES)()
    ret = lib.ipc_export_key(C.c_void_p(t.data_ptr()), buf)
    if ret:
        raise RuntimeError(f"ipc_export_key failed: {ret}")
    return bytes(buf)


def layer_keys(kv_caches) -> tuple[bytes, bytes | None]:
    """Concatenated K keys and V keys (None for a K-only cache) of per-layer
    tensors shaped [2, num_blocks, block_size, heads, head_dim] or
    [num_blocks, block_size, width] -- the k_raw_ptrs / v_raw_ptrs of a
    worker_context registered with per_len 72."""
    ks, vs = [], []
    for t in kv_caches:
        if t.dim() == 5:
            ks.append(ipckey_from_tensor(t[0]))
            vs.append(ipckey_from_tensor(t[1]))
        else:
            ks.append(ipckey_from_tensor(t))
    return b"".join(ks), (b"".join(vs) if vs else None)
