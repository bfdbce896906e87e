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

import struct

import torch

IPC_HANDLE_BYTES = 64
KEY_BYTES = IPC_HANDLE_BYTES + 8


def ipckey_from_tensor(t: torch.Tensor) -> bytes:
    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    st = t.untyped_storage()
    info = st._share_cuda_()
    handle, storage_offset_bytes = info[1], info[3]
    if len(handle) != IPC_HANDLE_BYTES:
        raise RuntimeError(f"unexpected IPC handle size {len(handle)}")
    off = storage_offset_bytes + t.storage_offset() * t.element_size()
    return bytes(handle) + struct.pack("<Q", off)


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
