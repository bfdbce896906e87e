"""ORACLE -- test infrastructure only.  numpy/ctypes front end of
kvcopy_oracle.c (the C restatement of CrossCache's CPU transfer path) and of
the reference's own compiled src/device/mem/mem.cpp (oracle/_ref).

The paged cache of one layer is a numpy uint8 array of
num_blocks * block_size * unit bytes (vLLM's [num_blocks, block_size, heads,
head_dim] layout flattened); a record is a uint8 array of
kv * num_layers * chunk_size * unit bytes.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_mem.so"


def _build_if_missing() -> None:
    if not LIB.exists():
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)


_build_if_missing()
_lib = C.CDLL(str(LIB))
_lib.oracle_slot_mapping.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
_lib.oracle_slot_mapping.restype = None
_lib.oracle_transfer.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint16,
                                 C.c_uint16, C.c_uint32, C.c_uint8, C.c_bool]
_lib.oracle_transfer.restype = C.c_int
_lib.oracle_cache_op.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                 C.c_uint32, C.c_uint32, C.c_uint16, C.c_uint32, C.c_uint8,
                                 C.c_bool, C.c_int]
_lib.oracle_cache_op.restype = C.c_int


def _ptrs(layers) -> np.ndarray:
    return np.array([a.ctypes.data for a in layers], dtype=np.uint64)


def slot_mapping(bids, block_size: int) -> np.ndarray:
    """cache.c:345-398: per-token slots of the blocks `bids`."""
    b = np.ascontiguousarray(np.asarray(bids, dtype=np.uint64))
    out = np.empty(len(b) * block_size, dtype=np.int64)
    _lib.oracle_slot_mapping(b.ctypes.data, len(b), block_size, out.ctypes.data)
    return out


def transfer(record: np.ndarray, k_layers, v_layers, slots: np.ndarray, num_tokens: int,
             hidden_dim_size: int, element_size: int, direction: bool) -> None:
    """mem.cpp:114-173 on one record (direction True: paged -> record)."""
    kp = _ptrs(k_layers)
    vp = _ptrs(v_layers) if v_layers is not None else None
    s = np.ascontiguousarray(slots, dtype=np.int64)
    _lib.oracle_transfer(record.ctypes.data, kp.ctypes.data, vp.ctypes.data if vp is not None else None,
                         s.ctypes.data, len(kp), num_tokens, hidden_dim_size, element_size, direction)


def cache_op(records, k_layers, v_layers, bids, chunk_size: int, block_size: int,
             hidden_dim_size: int, element_size: int, direction: bool, nthreads: int = 4) -> None:
    """cache.c:513-593 chunking: records[i] <-> blocks bids[i*bpc:(i+1)*bpc]."""
    kp = _ptrs(k_layers)
    vp = _ptrs(v_layers) if v_layers is not None else None
    recp = np.array([r.ctypes.data for r in records], dtype=np.uint64)
    b = np.ascontiguousarray(np.asarray(bids, dtype=np.uint64))
    _lib.oracle_cache_op(recp.ctypes.data, kp.ctypes.data, vp.ctypes.data if vp is not None else None,
                         b.ctypes.data, len(b), chunk_size, block_size, len(kp), hidden_dim_size,
                         element_size, direction, nthreads)


def gather(k_layers, v_layers, bids, chunk_size: int, block_size: int, unit: int,
           nthreads: int = 4) -> list[np.ndarray]:
    """Save: records for the chunks of `bids` (unit = hidden_dim_size * element_size bytes,
    passed as hidden_dim_size=unit, element_size=1 -- the copy is byte-exact)."""
    bpc = chunk_size // block_size
    kv = 2 if v_layers is not None else 1
    n = len(bids) // bpc
    recs = [np.zeros(kv * len(k_layers) * chunk_size * unit, dtype=np.uint8) for _ in range(n)]
    cache_op(recs, k_layers, v_layers, bids, chunk_size, block_size, unit, 1, True, nthreads)
    return recs


def scatter(records, k_layers, v_layers, bids, chunk_size: int, block_size: int, unit: int,
            nthreads: int = 4) -> None:
    """Load: write records into the blocks `bids` of the paged layers (in place)."""
    cache_op(records, k_layers, v_layers, bids, chunk_size, block_size, unit, 1, False, nthreads)


# ---------------------------------------------------------------------------
# the reference's own mem.cpp (oracle/_ref/libref_mem.so)

class _RefParams(C.Structure):
    _fields_ = [("caches", C.c_void_p), ("caches_h", C.c_void_p), ("keys_ptrs", C.c_void_p),
                ("value_ptrs", C.c_void_p), ("page_buffer_size", C.c_uint64),
                ("slot_mapping", C.c_void_p), ("devid", C.c_uint8),
                ("caches_element_size", C.c_uint8), ("num_layers", C.c_uint16),
                ("num_tokens", C.c_uint16), ("hidden_dim_size", C.c_uint32),
                ("direction", C.c_bool)]


class RefMem:
    """CrossCache's MemAdaptor::TransferKVCache, compiled from the reference
    sources.  It prints a line per token to stdout; calls are wrapped so that
    output goes to /dev/null."""

    def __init__(self, path: Path = REF_LIB):
        if not path.exists():
            raise FileNotFoundError(f"{path} (build with `make -C oracle ref` where the reference exists)")
        self.lib = C.CDLL(str(path))
        self.lib.mem_adaptor_create.restype = C.c_void_p
        self.lib.mem_adaptor_destroy.argtypes = [C.c_void_p]
        self.lib.transfer_kvcache.argtypes = [C.c_void_p, C.POINTER(_RefParams)]
        self.lib.transfer_kvcache.restype = C.c_int
        self.libc = C.CDLL(None)
        self.ad = self.lib.mem_adaptor_create()

    def close(self) -> None:
        if self.ad:
            self.lib.mem_adaptor_destroy(self.ad)
            self.ad = None

    def transfer(self, record: np.ndarray, k_layers, v_layers, slots: np.ndarray, num_tokens: int,
                 hidden_dim_size: int, element_size: int, direction: bool) -> int:
        kp = _ptrs(k_layers)
        vp = _ptrs(v_layers) if v_layers is not None else None
        s = np.ascontiguousarray(slots, dtype=np.int64)
        p = _RefParams(caches=record.ctypes.data, caches_h=record.ctypes.data,
                       keys_ptrs=kp.ctypes.data, value_ptrs=vp.ctypes.data if vp is not None else None,
                       page_buffer_size=0, slot_mapping=s.ctypes.data, devid=0,
                       caches_element_size=element_size, num_layers=len(kp), num_tokens=num_tokens,
                       hidden_dim_size=hidden_dim_size, direction=direction)
        sys.stdout.flush()
        saved = os.dup(1)
        devnull = os.open(os.devnull, os.O_WRONLY)
        try:
            os.dup2(devnull, 1)
            ret = self.lib.transfer_kvcache(self.ad, C.byref(p))
            self.libc.fflush(None)
        finally:
            os.dup2(saved, 1)
            os.close(saved)
            os.close(devnull)
        return ret
