"""Tensor-parallel agreement on the prefix-hit length.

Under TP each rank saves and loads its own KV-head shard in its own pool
(keyed (model, world_size, rank), CrossCache src/cache/cache.c:54-58), so a
key can be cached on one rank and evicted on another.  CrossCache answers
lookups from rank 0 only (src/main.c:135-136); here every rank looks up its
own map and one all-reduce(min) over the process group (NCCL over NVLink on
GPUs, gloo on CPU) gives every rank the same per-request hit count, so all
ranks load the same blocks.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def agree_min_hits(hits, group=None, device: torch.device | None = None) -> np.ndarray:
    """Element-wise minimum of the per-request hit counts over the group.

    hits: sequence / array of non-negative ints (one per request).  The
    collective runs on `device` (a CUDA device for NCCL) or on CPU (gloo).
    Every rank must call this with the same number of requests.
    """
    arr = np.asarray(hits, dtype=np.int32)
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return arr.copy()
    if device is None:
        backend = dist.get_backend(group)
        device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.from_numpy(arr.copy()).to(device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return t.cpu().numpy()


def head_shard(num_kv_heads: int, world_size: int, rank: int) -> tuple[int, int]:
    """[start, end) of the KV heads rank `rank` holds under TP world_size."""
    if num_kv_heads % world_size:
        raise ValueError("world size must divide the KV heads")
    per = num_kv_heads // world_size
    return rank * per, (rank + 1) * per
