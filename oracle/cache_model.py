"""ORACLE -- test infrastructure only.  Host-side cache semantics restated:

  lookup      CrossCache src/cache/cache.c:712-745 + src/main.c:140: walk the
              keys in order, a cached key refreshes its recency (key_access,
              :155-159), the first miss stops the walk; the C API returns
              hits * key_len, the server converts that to hits * chunk_size
              tokens.
  store       cache.c:513-593 + :495-504: one record per chunk key; a key
              already cached keeps its existing record.
  load        cache.c:558-569: memory hits refresh recency.
  eviction    deterministic LRU (the reference's policy is wall-clock based
              and unpinned, cache.c:291-343): when the pool is full a store
              takes the least-recently used record.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Sequence


class LRUPool:
    def __init__(self, capacity: int):
        self.capacity = capacity
        self.od: OrderedDict[bytes, None] = OrderedDict()   # first = least recent
        self.evictions = 0

    def lookup(self, keys: Sequence[bytes]) -> int:
        n = 0
        for k in keys:
            if k not in self.od:
                break
            self.od.move_to_end(k)
            n += 1
        return n

    def store(self, keys: Sequence[bytes]) -> list[bytes]:
        """returns the keys newly written (in order)"""
        new, pending = [], set()
        for k in keys:
            if k in self.od or k in pending:
                continue
            if len(self.od) + len(pending) >= self.capacity:
                if not self.od:
                    break           # everything pending: -ENOMEM
                self.od.popitem(last=False)
                self.evictions += 1
            pending.add(k)
            new.append(k)
        for k in new:               # published after the transfer, in key order
            self.od[k] = None
        return new

    def load(self, keys: Sequence[bytes]) -> list[bool]:
        hit = []
        for k in keys:
            if k in self.od:
                self.od.move_to_end(k)
                hit.append(True)
            else:
                hit.append(False)
        return hit

    def lru_order(self) -> list[bytes]:
        return list(self.od)
