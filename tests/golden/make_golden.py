"""Generate the committed golden fixtures (run where the reference exists):

    PYTHONPATH=. python tests/golden/make_golden.py

block_hashes.json  chained block hashes computed by the INSTALLED vLLM
                   (vllm.v1.core.kv_cache_utils.hash_block_tokens with
                   vllm.utils.hashing.sha256 and sha256_cbor, NONE_HASH from
                   init_none_hash under PYTHONHASHSEED=<seed>; some cases with
                   per-block extra_keys from gen.hash_extra) -- the function
                   CrossCache's keys come from
                   (python/crosscache_connector.py:133).
kv_records.json    SHA-256 digests of records gathered, and of paged layers
                   after a scatter, by CrossCache's own MemAdaptor::
                   TransferKVCache (src/device/mem/mem.cpp:114-173) compiled
                   from the reference sources into oracle/_ref/libref_mem.so
                   (`make -C oracle ref`), driven per chunk with the slot
                   mapping of src/cache/cache.c:345-398.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import numpy as np  # noqa: E402

from tests.golden import gen  # noqa: E402


def make_hashes() -> list[dict]:
    from vllm.utils.hashing import sha256, sha256_cbor
    from vllm.v1.core import kv_cache_utils as kcu

    out = []
    cases = [(i, c, "sha256", sha256) for i, c in enumerate(gen.HASH_CASES)]
    cases += [(100 + i, c, "sha256_cbor", sha256_cbor) for i, c in enumerate(gen.HASH_CASES_CBOR)]
    for i, (name, bs, seed, spec), algo, fn in cases:
        os.environ["PYTHONHASHSEED"] = seed
        kcu.init_none_hash(fn)
        tokens = gen.hash_tokens(spec, i)
        hashes = []
        parent = None
        for b in range(len(tokens) // bs):
            parent = kcu.hash_block_tokens(fn, parent, tokens[b * bs:(b + 1) * bs], None)
            hashes.append(bytes(parent).hex())
        out.append(dict(name=name, algo=algo, block_size=bs, pythonhashseed=seed,
                        none_hash=bytes(kcu.NONE_HASH).hex(), tokens=tokens, hashes=hashes))
    # extra keys: the per-block extra_keys tuples are regenerated from their
    # spec by tests/golden/gen.py hash_extra
    fns = {"sha256": sha256, "sha256_cbor": sha256_cbor}
    for i, (name, algo, bs, seed, spec, xspec) in enumerate(gen.HASH_CASES_EXTRA):
        os.environ["PYTHONHASHSEED"] = seed
        kcu.init_none_hash(fns[algo])
        tokens = gen.hash_tokens(spec, 200 + i)
        extra = gen.hash_extra(xspec, len(tokens) // bs)
        hashes = []
        parent = None
        for b in range(len(tokens) // bs):
            parent = kcu.hash_block_tokens(fns[algo], parent, tokens[b * bs:(b + 1) * bs], extra[b])
            hashes.append(bytes(parent).hex())
        out.append(dict(name=name, algo=algo, block_size=bs, pythonhashseed=seed,
                        none_hash=bytes(kcu.NONE_HASH).hex(), tokens=tokens, extra=xspec, hashes=hashes))
    return out


def make_records() -> list[dict]:
    from oracle.kvcopy import RefMem, slot_mapping

    ref = RefMem()
    out = []
    for case in gen.KV_CASES:
        k, v = gen.paged_layers(case)
        bids = gen.block_ids(case)
        bpc = case["chunk_size"] // case["block_size"]
        rec_sha = []
        for c in range(case["chunks"]):
            rec = np.zeros(gen.record_bytes(case), np.uint8)
            slots = slot_mapping(bids[c * bpc:(c + 1) * bpc], case["block_size"])
            assert ref.transfer(rec, k, v, slots, case["chunk_size"], case["hidden"], case["elt"], True) == 0
            rec_sha.append(gen.sha(rec))
        # scatter seeded records into zeroed layers at a second block table
        k0, v0 = gen.paged_layers(case, zero=True)
        bids2 = gen.block_ids(case, seed_offset=1)
        for c, rec in enumerate(gen.records_for_scatter(case)):
            slots = slot_mapping(bids2[c * bpc:(c + 1) * bpc], case["block_size"])
            assert ref.transfer(rec, k0, v0, slots, case["chunk_size"], case["hidden"], case["elt"], False) == 0
        out.append(dict(case=case["name"], bids=bids.tolist(), record_sha256=rec_sha,
                        scatter_bids=bids2.tolist(),
                        scatter_k_sha256=[gen.sha(a) for a in k0],
                        scatter_v_sha256=[gen.sha(a) for a in v0] if v0 is not None else None))
    ref.close()
    return out


def main() -> None:
    (HERE / "block_hashes.json").write_text(json.dumps(make_hashes(), indent=1) + "\n")
    (HERE / "kv_records.json").write_text(json.dumps(make_records(), indent=1) + "\n")
    print("wrote", HERE / "block_hashes.json", HERE / "kv_records.json")


if __name__ == "__main__":
    main()
