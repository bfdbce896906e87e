"""ORACLE -- test infrastructure only.  Restatement of vLLM's default prefix
block hash, the key CrossCache stores records under:

  vllm/v1/core/kv_cache_utils.py:541-570  hash_block_tokens:
      h_i = hash_fn((parent or NONE_HASH, tuple(block tokens), extra_keys))
  vllm/utils/hashing.py:26-41  sha256: SHA-256 of pickle.dumps(obj, protocol=5)
  vllm/v1/core/kv_cache_utils.py:97-112  init_none_hash:
      NONE_HASH = hash_fn(PYTHONHASHSEED string)
  CrossCache python/adaptor.py:32-40  striding_block_hashes: chunk keys are
      the hashes of blocks bpc-1, 2*bpc-1, ...
  vllm/utils/hashing.py:43-57  sha256_cbor: SHA-256 of cbor2.dumps(obj,
      canonical=True) -- the same triple as a CBOR array (RFC 8949: shortest
      heads, definite lengths)

The pickle byte stream is written out here opcode by opcode (CPython
_pickle.c: PROTO, FRAME, SHORT_BINBYTES, MEMOIZE, MARK, BININT1/BININT2/
BININT, TUPLE or TUPLE1..3, NONE, TUPLE3, STOP) instead of calling pickle, so
that this file states the exact bytes the device kernel must produce; tests
check it against pickle and against golden vectors produced by vLLM itself.
"""
from __future__ import annotations

import hashlib
import struct
from typing import Iterable, Sequence

PROTO, FRAME, SHORT_BINBYTES, MEMOIZE, MARK = 0x80, 0x95, 0x43, 0x94, 0x28
BININT1, BININT2, BININT, TUPLE, NONE, TUPLE3, STOP = 0x4B, 0x4D, 0x4A, 0x74, 0x4E, 0x87, 0x2E
TUPLE_N = {1: 0x85, 2: 0x86, 3: 0x87}


def _int_op(v: int) -> bytes:
    if 0 <= v <= 0xFF:
        return bytes([BININT1, v])
    if 0 <= v <= 0xFFFF:
        return bytes([BININT2]) + struct.pack("<H", v)
    if -0x80000000 <= v <= 0x7FFFFFFF:
        return bytes([BININT]) + struct.pack("<i", v)
    raise ValueError("token id outside int32")


def pickle_block(parent: bytes, tokens: Sequence[int]) -> bytes:
    """pickle.dumps((parent, tuple(tokens), None), protocol=5) for a 32-byte
    parent and 1 <= len(tokens) <= 8192 (a single pickle frame)."""
    if len(parent) != 32 or not 1 <= len(tokens) <= 8192:
        raise ValueError("unsupported block")
    body = bytearray([SHORT_BINBYTES, 32]) + parent + bytes([MEMOIZE])
    n = len(tokens)
    if n > 3:
        body.append(MARK)
    for v in tokens:
        body += _int_op(int(v))
    body.append(TUPLE if n > 3 else TUPLE_N[n])
    body += bytes([MEMOIZE, NONE, TUPLE3, MEMOIZE, STOP])
    return bytes([PROTO, 5, FRAME]) + struct.pack("<Q", len(body)) + bytes(body)


def _cbor_head(major: int, n: int) -> bytes:
    """RFC 8949 shortest head for major type `major` and argument n"""
    if n < 24:
        return bytes([major << 5 | n])
    if n < 0x100:
        return bytes([major << 5 | 24, n])
    if n < 0x10000:
        return bytes([major << 5 | 25]) + struct.pack(">H", n)
    if n < 0x100000000:
        return bytes([major << 5 | 26]) + struct.pack(">I", n)
    return bytes([major << 5 | 27]) + struct.pack(">Q", n)


def cbor_block(parent: bytes, tokens: Sequence[int]) -> bytes:
    """cbor2.dumps((parent, tuple(tokens), None), canonical=True) for int32 tokens"""
    if len(parent) != 32:
        raise ValueError("parent must be 32 bytes")
    out = bytearray(_cbor_head(4, 3)) + _cbor_head(2, 32) + parent + _cbor_head(4, len(tokens))
    for v in tokens:
        v = int(v)
        if not -0x80000000 <= v <= 0x7FFFFFFF:
            raise ValueError("token id outside int32")
        out += _cbor_head(0, v) if v >= 0 else _cbor_head(1, -1 - v)
    out.append(0xF6)                      # simple value null
    return bytes(out)


def none_hash(seed: str, algo: str = "sha256") -> bytes:
    """NONE_HASH for PYTHONHASHSEED=seed: hash_fn(seed) -- sha256 of
    pickle.dumps(seed, 5), or sha256 of the canonical CBOR text string."""
    b = seed.encode()
    if algo == "sha256_cbor":
        return hashlib.sha256(_cbor_head(3, len(b)) + b).digest()
    if len(b) >= 256:
        raise ValueError("seed too long for this restatement")
    # PROTO 5, FRAME, SHORT_BINUNICODE len data, MEMOIZE, STOP
    body = bytes([0x8C, len(b)]) + b + bytes([MEMOIZE, STOP])
    msg = bytes([PROTO, 5, FRAME]) + struct.pack("<Q", len(body)) + body
    return hashlib.sha256(msg).digest()


def serialise_with_extra(parent: bytes, tokens: Sequence[int], extra, algo: str = "sha256") -> bytes:
    """vLLM's hash input with extra keys, by definition: hash_fn's own
    serialiser applied to (parent, tuple(tokens), extra_keys)
    (vllm/utils/hashing.py sha256 / sha256_cbor)."""
    obj = (parent, tuple(int(t) for t in tokens), extra)
    if algo == "sha256_cbor":
        import cbor2
        return cbor2.dumps(obj, canonical=True)
    import pickle
    return pickle.dumps(obj, protocol=5)


def block_hashes(tokens: Sequence[int], block_size: int, parent: bytes, algo: str = "sha256",
                 extra: Sequence | None = None) -> list[bytes]:
    """Chained hashes of the full blocks of `tokens` starting from `parent`;
    extra[i] (optional) is block i's extra_keys tuple or None."""
    ser = cbor_block if algo == "sha256_cbor" else pickle_block
    out = []
    h = parent
    for i in range(len(tokens) // block_size):
        blk = tokens[i * block_size:(i + 1) * block_size]
        if extra is not None and extra[i] is not None:
            msg = serialise_with_extra(h, blk, extra[i], algo)
        else:
            msg = ser(h, blk)
        h = hashlib.sha256(msg).digest()
        out.append(h)
    return out


def chunk_keys(hashes: Sequence[bytes], blocks_in_chunk: int) -> list[bytes]:
    """python/adaptor.py:32-40 striding_block_hashes."""
    return list(hashes[blocks_in_chunk - 1::blocks_in_chunk])


def batch_block_hashes(requests: Iterable[Sequence[int]], block_size: int, parent: bytes,
                       algo: str = "sha256", extra: Sequence | None = None) -> list[list[bytes]]:
    reqs = list(requests)
    return [block_hashes(t, block_size, parent, algo, extra[r] if extra is not None else None)
            for r, t in enumerate(reqs)]
