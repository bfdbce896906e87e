"""ORACLE -- test infrastructure only.

CPU restatements of CrossCache's hot path used as the parity checker by
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs.
Nothing in the demo_b200 product package imports this package.

  kvcopy.py       record gather/scatter: C restatement (liboracle.so) of
                  src/device/mem/mem.cpp:114-173 + src/cache/cache.c:345-398,
                  513-593, and a loader for the reference's own mem.cpp
                  compiled into _ref/libref_mem.so (Makefile target `ref`)
  blockhash.py    vLLM's chained sha256 block hash (pickle protocol 5 framing
                  restated byte by byte + hashlib SHA-256)
  cache_model.py  prefix lookup (cache.c:712-745) and a deterministic LRU
                  record-pool model
"""

import os as _os
from pathlib import Path as _Path

REFERENCE_ENV = "CROSSCACHE_REFERENCE"


def reference_root() -> _Path:
    """The CrossCache source tree the checker builds and reads (the reference
    project's CrossCache/ directory): $CROSSCACHE_REFERENCE, else where this
    build's container mounts it.  May not exist (it never does on a GPU
    box): callers check .exists()."""
    return _Path(_os.environ.get(REFERENCE_ENV, "/root/reference/CrossCache"))
