"""Client <-> server messages of CrossCache, byte-compatible with the
reference (include/inner_h/protocol.h:1-67 for the layout, the encoder in
python/utils/protocol.py:125-255, the decoder in src/main.c:244-347).

Every message is one ZeroMQ frame: a 12-byte header (version, op, node_id,
reserved, len = body bytes, uid), little-endian and packed, then the body:

  REGISTER    world_size, rank_id, num_layers, kv_flags, num_blocks,
              block_size, hidden_dim_size, first_key_in_bytes (20 bytes),
              model name + NUL, the K keys of every layer, then the V keys
              (absent when kv_flags has no K_V_MASK bit: a K-only cache)
  UNREGISTER  empty body
  LOOKUP      keys_num, key_len, keys, world_size (1 byte), model name + NUL
  STORE/LOAD  keys_num, key_len, keys, then uint64 block ids to the end
  response    uid, ok (uint32; a negative errno in two's complement, or the
              number of hit tokens for a lookup)

The encoder produces the reference client's bytes exactly, including its
version field (1 on REGISTER, left 0 on the others; the server checks it on
REGISTER only, main.c:257-261, as decode_request does here).  Differences:
UNREGISTER encodes (the reference encoder returns None for it, so its
unregister cannot be sent); decode_request checks every length against the
frame instead of trusting them; a REGISTER of a worker whose planes are not
dense token-major (vLLM FlashInfer) ends with a 16-byte paged-geometry
trailer after the keys (b"PGEO", uint64 block_stride, uint32 head_bytes),
sent only for such workers, so a dense worker's REGISTER is the reference's.
"""
from __future__ import annotations

import enum
import struct
from dataclasses import dataclass

import numpy as np

CACHE_VERSION = 1
K_V_MASK = 0x01
KV_DTYPE_1BYTE = 0x02
KV_DTYPE_2BYTE = 0x04
KV_DTYPE_4BYTE = 0x08


class Op(enum.IntEnum):
    REGISTER = 0
    UNREGISTER = 1
    LOOKUP = 2
    STORE = 3
    LOAD = 4
    GET_INFO = 5


HEADER = struct.Struct("<BBBBII")       # msg_header
REGISTER = struct.Struct("<BBBBIIII")   # msg_register
COMMON = struct.Struct("<II")           # msg_common
LOOKUP_TAIL = struct.Struct("<B")       # msg_lookup
RESPONSE = struct.Struct("<II")         # msg_response
GEOMETRY = struct.Struct("<4sQI")       # REGISTER trailer of a non-dense worker
GEOMETRY_MAGIC = b"PGEO"


class ProtocolError(ValueError):
    pass


def kv_flags(has_v: bool, element_size: int) -> int:
    """python/utils/protocol.py:15-21 (unknown sizes are sent as 2 bytes)"""
    f = K_V_MASK if has_v else 0
    return f | {1: KV_DTYPE_1BYTE, 4: KV_DTYPE_4BYTE}.get(element_size, KV_DTYPE_2BYTE)


def element_size_of(flags: int) -> int:
    """main.c:231-240 dtype_to_bytes"""
    if flags & KV_DTYPE_1BYTE:
        return 1
    if flags & KV_DTYPE_2BYTE:
        return 2
    if flags & KV_DTYPE_4BYTE:
        return 4
    return 2


@dataclass
class Register:
    node_id: int
    uid: int
    world_size: int
    rank_id: int
    num_blocks: int
    block_size: int
    element_size: int
    hidden_dim_size: int
    key_len: int                  # first_key_in_bytes: bytes of one layer's key
    model_name: str
    k_keys: bytes                 # num_layers * key_len
    v_keys: bytes | None          # same, or None for a K-only cache
    version: int = CACHE_VERSION
    block_stride: int = 0         # paged geometry trailer (0 / 0: dense)
    head_bytes: int = 0

    @property
    def num_layers(self) -> int:
        return len(self.k_keys) // self.key_len if self.key_len else 0


@dataclass
class Unregister:
    node_id: int
    uid: int


@dataclass
class Lookup:
    node_id: int
    uid: int
    keys: bytes
    keys_num: int
    key_len: int
    world_size: int
    model_name: str


@dataclass
class Transfer:
    op: Op                        # STORE or LOAD
    node_id: int
    uid: int
    keys: bytes
    keys_num: int
    key_len: int
    block_ids: np.ndarray         # uint64


def _header(op: int, node_id: int, uid: int, body_len: int) -> bytes:
    version = CACHE_VERSION if op == Op.REGISTER else 0
    return HEADER.pack(version, int(op), node_id & 0xFF, 0, body_len, uid & 0xFFFFFFFF)


def _name(s: str) -> bytes:
    b = s.encode("utf-8")
    if b"\0" in b:
        raise ProtocolError("model name contains NUL")
    return b + b"\0"


def _keys(keys) -> tuple[bytes, int, int]:
    if isinstance(keys, (bytes, bytearray, memoryview)):
        raise ProtocolError("keys must be a sequence of per-key byte strings")
    keys = [bytes(k) for k in keys]
    klen = len(keys[0]) if keys else 0
    if any(len(k) != klen for k in keys):
        raise ProtocolError("keys must all have the same length")
    return b"".join(keys), len(keys), klen


def encode_register(node_id: int, uid: int, world_size: int, rank_id: int, num_blocks: int,
                    block_size: int, element_size: int, hidden_dim_size: int, key_len: int,
                    model_name: str, layer_keys: list[tuple[bytes, ...]], block_stride: int = 0,
                    head_bytes: int = 0) -> bytes:
    """layer_keys: per layer (k_key,) or (k_key, v_key), each key_len bytes
    (python/utils/protocol.py:125-180: K keys of every layer, then V keys).
    A non-zero block_stride / head_bytes appends the geometry trailer."""
    if not layer_keys:
        raise ProtocolError("no layers")
    has_v = len(layer_keys[0]) > 1
    if len(layer_keys) > 255:
        raise ProtocolError("num_layers is one byte on the wire")
    for lk in layer_keys:
        if len(lk) != len(layer_keys[0]) or any(len(k) != key_len for k in lk):
            raise ProtocolError(f"every layer key must be {key_len} bytes")
    body = REGISTER.pack(world_size, rank_id, len(layer_keys), kv_flags(has_v, element_size),
                         num_blocks, block_size, hidden_dim_size, key_len)
    body += _name(model_name) + b"".join(lk[0] for lk in layer_keys)
    if has_v:
        body += b"".join(lk[1] for lk in layer_keys)
    if block_stride or head_bytes:
        body += GEOMETRY.pack(GEOMETRY_MAGIC, block_stride, head_bytes)
    return _header(Op.REGISTER, node_id, uid, len(body)) + body


def encode_unregister(node_id: int, uid: int) -> bytes:
    return _header(Op.UNREGISTER, node_id, uid, 0)


def encode_lookup(node_id: int, uid: int, keys, world_size: int, model_name: str) -> bytes:
    kb, n, klen = _keys(keys)
    body = COMMON.pack(n, klen) + kb + LOOKUP_TAIL.pack(world_size) + _name(model_name)
    return _header(Op.LOOKUP, node_id, uid, len(body)) + body


def encode_transfer(op: Op, node_id: int, uid: int, keys, block_ids) -> bytes:
    if op not in (Op.STORE, Op.LOAD):
        raise ProtocolError("STORE or LOAD")
    kb, n, klen = _keys(keys)
    bids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.uint64)).astype("<u8", copy=False)
    body = COMMON.pack(n, klen) + kb + bids.tobytes()
    return _header(op, node_id, uid, len(body)) + body


def encode_response(uid: int, ret: int) -> bytes:
    return RESPONSE.pack(uid & 0xFFFFFFFF, ret & 0xFFFFFFFF)


def decode_response(frame: bytes) -> tuple[int, int]:
    """(uid, status as a signed 32-bit value)"""
    if len(frame) < RESPONSE.size:
        raise ProtocolError("short response")
    uid, ok = RESPONSE.unpack_from(frame)
    return uid, ok - (1 << 32) if ok >= 1 << 31 else ok


def _cstr(buf: bytes, pos: int) -> tuple[str, int]:
    end = buf.find(b"\0", pos)
    if end < 0:
        raise ProtocolError("unterminated model name")
    return buf[pos:end].decode("utf-8", errors="replace"), end + 1


def decode_request(frame: bytes):
    """One request frame -> Register | Unregister | Lookup | Transfer.
    Raises ProtocolError (with .uid when the header was readable)."""
    if len(frame) < HEADER.size:
        raise ProtocolError("short header")
    version, op, node_id, _, blen, uid = HEADER.unpack_from(frame)
    body = memoryview(frame)[HEADER.size:]

    def fail(why):
        e = ProtocolError(why)
        e.uid = uid
        return e

    if blen != len(body):
        raise fail(f"header len {blen} != body {len(body)}")
    body = bytes(body)
    try:
        op = Op(op)
    except ValueError:
        raise fail(f"unknown op {op}") from None
    if op == Op.REGISTER:
        if version != CACHE_VERSION:
            raise fail(f"version {version}")
        if len(body) < REGISTER.size:
            raise fail("short register body")
        ws, rank, nl, flags, nb, bs, hid, klen = REGISTER.unpack_from(body)
        name, pos = _cstr(body, REGISTER.size)
        nk = 2 if flags & K_V_MASK else 1
        kend = pos + nk * nl * klen
        stride = hb = 0
        if nl and klen and len(body) == kend + GEOMETRY.size and body[kend:kend + 4] == GEOMETRY_MAGIC:
            _, stride, hb = GEOMETRY.unpack_from(body, kend)
        elif not nl or not klen or len(body) != kend:
            raise fail("register keys do not match num_layers * first_key_in_bytes")
        kk = body[pos:pos + nl * klen]
        vk = body[pos + nl * klen:kend] if nk == 2 else None
        return Register(node_id, uid, ws, rank, nb, bs, element_size_of(flags), hid, klen, name, kk, vk,
                        version, stride, hb)
    if op == Op.UNREGISTER:
        return Unregister(node_id, uid)
    if op in (Op.LOOKUP, Op.STORE, Op.LOAD):
        if len(body) < COMMON.size:
            raise fail("short body")
        n, klen = COMMON.unpack_from(body)
        kend = COMMON.size + n * klen
        if kend > len(body):
            raise fail("keys past the end of the message")
        keys = body[COMMON.size:kend]
        if op == Op.LOOKUP:
            if kend + LOOKUP_TAIL.size > len(body):
                raise fail("short lookup tail")
            (ws,) = LOOKUP_TAIL.unpack_from(body, kend)
            name, _ = _cstr(body, kend + LOOKUP_TAIL.size)
            return Lookup(node_id, uid, keys, n, klen, ws, name)
        rest = len(body) - kend
        if rest % 8:
            raise fail("block ids are not whole uint64s")
        bids = np.frombuffer(body, dtype="<u8", count=rest // 8, offset=kend).astype(np.uint64)
        return Transfer(op, node_id, uid, keys, n, klen, bids)
    raise fail(f"op {op.name} is not served")
