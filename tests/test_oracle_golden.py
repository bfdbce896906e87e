"""Pin the oracle: the CPU restatements against the golden vectors produced by
the installed vLLM hasher and by CrossCache's own compiled mem.cpp."""
import hashlib
import pickle
import random
import struct

import numpy as np
import pytest

from oracle import blockhash as bh
from oracle import kvcopy as ok
from tests.golden import gen


def test_hash_restatement_matches_vllm_golden(golden_hashes):
    assert len(golden_hashes) == len(gen.HASH_CASES) + len(gen.HASH_CASES_CBOR) + len(gen.HASH_CASES_EXTRA)
    assert {c["algo"] for c in golden_hashes} == {"sha256", "sha256_cbor"}
    for case in golden_hashes:
        nh = bytes.fromhex(case["none_hash"])
        assert nh == bh.none_hash(case["pythonhashseed"], case["algo"]), case["name"]
        extra = (gen.hash_extra(case["extra"], len(case["tokens"]) // case["block_size"])
                 if "extra" in case else None)
        got = bh.block_hashes(case["tokens"], case["block_size"], nh, case["algo"], extra)
        assert [h.hex() for h in got] == case["hashes"], case["name"]


@pytest.mark.parametrize("algo", ["sha256", "sha256_cbor"])
def test_extra_key_segments_splice_into_the_none_byte(algo, golden_hashes):
    """the segment demo_b200.hashing.extra_segment hands the kernel, put in
    place of None, gives the hash function's own serialisation"""
    from demo_b200.hashing import extra_segment

    par = bytes(range(32))
    n = 0
    for case in golden_hashes:
        if case.get("extra") is None or case["algo"] != algo:
            continue
        bs = case["block_size"]
        toks = case["tokens"]
        for i, ek in enumerate(gen.hash_extra(case["extra"], len(toks) // bs)):
            blk = toks[i * bs:(i + 1) * bs]
            seg = extra_segment(ek, algo)
            if ek is None:
                assert seg == b""
                continue
            if algo == "sha256_cbor":
                spliced = bh.cbor_block(par, blk)[:-1] + seg
            else:
                base = bh.pickle_block(par, blk)
                body = base[11:-4] + seg + base[-3:]
                spliced = base[:3] + struct.pack("<Q", len(body)) + body
            assert spliced == bh.serialise_with_extra(par, blk, ek, algo), (case["name"], i)
            n += 1
    assert n > 10


@pytest.mark.parametrize("bs", [1, 3, 16, 23, 24, 255, 256, 300])
def test_cbor_block_bytes_equal_cbor2(bs):
    cbor2 = pytest.importorskip("cbor2")
    rnd = random.Random(1000 + bs)
    for lo, hi in [(0, 24), (0, 256), (0, 65536), (0, 128256), (-2**31, 2**31)]:
        toks = [rnd.randrange(lo, hi) for _ in range(bs)]
        parent = bytes(rnd.randrange(256) for _ in range(32))
        assert bh.cbor_block(parent, toks) == cbor2.dumps((parent, tuple(toks), None), canonical=True)


def test_golden_tokens_cover_pickle_int_widths(golden_hashes):
    toks = [t for c in golden_hashes for t in c["tokens"]]
    assert any(0 <= t <= 255 for t in toks)
    assert any(256 <= t <= 65535 for t in toks)
    assert any(t >= 65536 for t in toks)
    assert any(t < 0 for t in toks)
    assert {c["block_size"] for c in golden_hashes} >= {1, 2, 3, 4, 16, 64}


@pytest.mark.parametrize("bs", [1, 2, 3, 4, 7, 16, 64, 257])
def test_pickle_block_bytes_equal_cpython(bs):
    rnd = random.Random(bs)
    for lo, hi in [(0, 256), (0, 65536), (0, 128256), (-2**31, 2**31)]:
        toks = [rnd.randrange(lo, hi) for _ in range(bs)]
        parent = bytes(rnd.randrange(256) for _ in range(32))
        assert bh.pickle_block(parent, toks) == pickle.dumps((parent, tuple(toks), None), protocol=5)


def test_chunk_key_striding():
    hs = [bytes([i]) * 32 for i in range(40)]
    assert bh.chunk_keys(hs, 16) == [hs[15], hs[31]]
    assert bh.chunk_keys(hs[:15], 16) == []


@pytest.mark.parametrize("case", gen.KV_CASES, ids=lambda c: c["name"])
def test_kvcopy_restatement_matches_reference_golden(case, golden_records):
    g = golden_records[case["name"]]
    k, v = gen.paged_layers(case)
    bids = gen.block_ids(case)
    assert bids.tolist() == g["bids"]
    recs = ok.gather(k, v, bids, case["chunk_size"], case["block_size"], gen.unit_of(case))
    assert [gen.sha(r) for r in recs] == g["record_sha256"]

    k0, v0 = gen.paged_layers(case, zero=True)
    bids2 = gen.block_ids(case, seed_offset=1)
    ok.scatter(gen.records_for_scatter(case), k0, v0, bids2, case["chunk_size"], case["block_size"],
               gen.unit_of(case))
    assert [gen.sha(a) for a in k0] == g["scatter_k_sha256"]
    if v0 is not None:
        assert [gen.sha(a) for a in v0] == g["scatter_v_sha256"]


def test_kvcopy_restatement_matches_compiled_reference_random():
    """Extra cases straight against the reference's own mem.cpp, when built."""
    if not ok.REF_LIB.exists():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    ref = ok.RefMem()
    rng = np.random.default_rng(3)
    for trial in range(4):
        L, hidden, elt, C = 3, int(rng.integers(1, 40)), int(rng.choice([1, 2, 4])), 12
        nb, bs = 20, 3
        unit = hidden * elt
        k = [rng.integers(0, 256, nb * bs * unit, dtype=np.uint8) for _ in range(L)]
        v = [rng.integers(0, 256, nb * bs * unit, dtype=np.uint8) for _ in range(L)]
        slots = rng.permutation(nb * bs)[:C].astype(np.int64)   # arbitrary per-token slots
        r1 = np.zeros(2 * L * C * unit, np.uint8)
        r2 = np.zeros_like(r1)
        assert ref.transfer(r1, k, v, slots, C, hidden, elt, True) == 0
        ok.transfer(r2, k, v, slots, C, hidden, elt, True)
        assert np.array_equal(r1, r2), trial
    ref.close()


def test_record_layout_explicit_small():
    """The record layout spelled out by hand: K[l][t] then V[l][t]."""
    L, C, unit, bs, nb = 2, 4, 3, 2, 5
    k = [np.arange(nb * bs * unit, dtype=np.uint8) + 10 * l for l in range(L)]
    v = [np.arange(nb * bs * unit, dtype=np.uint8) + 100 + 10 * l for l in range(L)]
    bids = np.array([3, 1], dtype=np.uint64)
    rec = ok.gather(k, v, bids, C, bs, unit)[0]
    slots = [3 * bs, 3 * bs + 1, 1 * bs, 1 * bs + 1]
    exp = []
    for layers in (k, v):
        for l in range(L):
            for s in slots:
                exp.extend(layers[l][s * unit:(s + 1) * unit])
    assert rec.tolist() == exp
    assert hashlib.sha256(rec.tobytes()).hexdigest() == gen.sha(np.array(exp, np.uint8))
