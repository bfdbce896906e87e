"""Device block hashing (include/kvhash.h) for torch token tensors.

block_hashes() returns the same bytes as vLLM's hash_block_tokens with the
sha256 or sha256_cbor hash function (vllm/v1/core/kv_cache_utils.py:541-570,
vllm/utils/hashing.py:26-57) for every full block of every request; chunk_keys() strides them the way CrossCache's
adaptor does (python/adaptor.py:32-40).
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
from typing import Sequence

import torch

from ._lib import KVHASH_ALGOS, lib


def none_hash_for_seed(seed: str | None = None, algo: str = "sha256") -> bytes:
    """NONE_HASH as vLLM's init_none_hash derives it from PYTHONHASHSEED
    (kv_cache_utils.py:97-112): the hash function applied to the seed string
    (pickled for "sha256", canonical CBOR for "sha256_cbor"); random when no
    seed is set."""
    import pickle

    seed = os.getenv("PYTHONHASHSEED") if seed is None else seed
    if seed is None:
        return os.urandom(32)
    if algo == "sha256_cbor":
        import cbor2
        return hashlib.sha256(cbor2.dumps(seed, canonical=True)).digest()
    return hashlib.sha256(pickle.dumps(seed, protocol=pickle.HIGHEST_PROTOCOL)).digest()


def block_hashes_device(tokens: torch.Tensor, tok_offsets: torch.Tensor, num_blocks: torch.Tensor,
                        out_offsets: torch.Tensor, block_size: int, none_hash: bytes,
                        out: torch.Tensor, parents: torch.Tensor | None = None,
                        stream: torch.cuda.Stream | None = None, algo: str = "sha256") -> None:
    """Launch the hash kernel on device tensors (int32 tokens, int64 offsets,
    int32 block counts, uint8 [total, 32] output).  Asynchronous."""
    for t, dt in ((tokens, torch.int32), (tok_offsets, torch.int64), (num_blocks, torch.int32),
                  (out_offsets, torch.int64), (out, torch.uint8)):
        if t.dtype != dt or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"expected contiguous CUDA {dt}")
    if len(none_hash) != 32:
        raise ValueError("none_hash must be 32 bytes")
    s = stream if stream is not None else torch.cuda.current_stream(tokens.device)
    ret = lib.kv_block_hash_launch_algo(tokens.data_ptr(), tok_offsets.data_ptr(), num_blocks.data_ptr(),
                                        out_offsets.data_ptr(),
                                        parents.data_ptr() if parents is not None else None,
                                        tok_offsets.numel(), block_size, none_hash, out.data_ptr(),
                                        KVHASH_ALGOS[algo], C.c_void_p(s.cuda_stream))
    if ret:
        raise RuntimeError(f"kv_block_hash_launch failed: {ret}")


_FRAME_LIMIT = 1 << 16      # pickle protocol 5 commits a new frame past 64 KiB


def extra_segment(extra_keys, algo: str = "sha256") -> bytes:
    """The bytes extra_keys occupy inside the serialised (parent, tokens,
    extra_keys) tuple -- what include/kvhash.h's _ext entry points splice in
    place of the None byte.  Taken from the hash function's own serialiser
    (pickle protocol 5 / canonical CBOR) on a template tuple; protocol 5
    memoizes without indices and CBOR has no back-references, so the segment
    does not depend on where it sits.  b"" for None."""
    if extra_keys is None:
        return b""
    parent = bytes(32)
    if algo == "sha256_cbor":
        import cbor2
        base = cbor2.dumps((parent, (0,), None), canonical=True)
        full = cbor2.dumps((parent, (0,), extra_keys), canonical=True)
        if full[:len(base) - 1] != base[:-1]:
            raise ValueError("unexpected CBOR layout")
        return full[len(base) - 1:]
    import pickle
    base = pickle.dumps((parent, (0,), None), protocol=5)
    full = pickle.dumps((parent, (0,), extra_keys), protocol=5)
    cut = len(base) - 4                     # NONE, then TUPLE3 MEMOIZE STOP
    if (full[:3] != base[:3] or full[11:cut] != base[11:cut] or full[-3:] != base[-3:]
            or len(full) >= _FRAME_LIMIT):
        raise ValueError("extra keys do not serialise as one pickle frame segment")
    return full[cut:len(full) - 3]


def block_hashes(token_lists: Sequence[Sequence[int]], block_size: int, none_hash: bytes,
                 device: int = 0, algo: str = "sha256",
                 extra_keys: Sequence[Sequence] | None = None) -> list[list[bytes]]:
    """Chained block hashes of each request (host lists in, host bytes out),
    computed on `device` through kv_block_hash_host_ext.  extra_keys[r][i]
    (optional) is request r's block i extra_keys tuple, or None, as vLLM's
    generate_block_hash_extra_keys returns it."""
    import numpy as np

    lens = np.array([len(t) for t in token_lists], dtype=np.int64)
    flat = np.ascontiguousarray(np.concatenate([np.asarray(t, dtype=np.int64) for t in token_lists])
                                if len(token_lists) else np.zeros(0, np.int64))
    if flat.size and (flat.min() < -2**31 or flat.max() >= 2**31):
        raise ValueError("token ids must fit in int32")
    flat = flat.astype(np.int32)
    nblk = lens // block_size
    out = np.zeros((int(nblk.sum()), 32), dtype=np.uint8)
    xbuf = xoff = None
    if extra_keys is not None:
        segs = []
        for r, n in enumerate(nblk):
            ek = extra_keys[r] if extra_keys[r] is not None else [None] * int(n)
            if len(ek) < n:
                raise ValueError("one extra_keys entry per full block")
            for i in range(int(n)):
                s = extra_segment(ek[i], algo)
                if algo == "sha256" and 47 + 5 * block_size + 6 + len(s) >= _FRAME_LIMIT:
                    raise ValueError("block with extra keys does not fit one pickle frame")
                segs.append(s)
        xoff = np.zeros(len(segs) + 1, dtype=np.int64)
        xoff[1:] = np.cumsum([len(s) for s in segs])
        xbuf = np.frombuffer(b"".join(segs) or b"\0", dtype=np.uint8).copy()
    ret = lib.kv_block_hash_host_ext(device, flat.ctypes.data, lens.ctypes.data, len(lens), block_size,
                                     none_hash, xbuf.ctypes.data if xbuf is not None else None,
                                     xoff.ctypes.data if xoff is not None else None, out.ctypes.data,
                                     KVHASH_ALGOS[algo])
    if ret < 0:
        raise RuntimeError(f"kv_block_hash_host failed: {ret}")
    res, off = [], 0
    for n in nblk:
        res.append([bytes(out[off + i]) for i in range(int(n))])
        off += int(n)
    return res


def chunk_keys(hashes: Sequence[bytes], blocks_in_chunk: int) -> list[bytes]:
    """Every blocks_in_chunk-th hash (CrossCache python/adaptor.py:32-40)."""
    return list(hashes[blocks_in_chunk - 1::blocks_in_chunk])
