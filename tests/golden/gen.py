"""Seeded input generators shared by make_golden.py and the tests.

Every paged layer and record is a deterministic function of a seed (numpy
PCG64), so fixtures store only seeds, shapes and SHA-256 digests of outputs.
"""
from __future__ import annotations

import hashlib

import numpy as np

# cases pinned by make_golden.py (names are stable fixture keys)
KV_CASES = [
    # CrossCache tests/test_copy.cpp:95-105 defaults: 40 blocks of 2 tokens,
    # 4-token chunks, 2 layers, hidden 4096, 2-byte elements, K and V
    dict(name="test_copy_defaults", num_blocks=40, block_size=2, chunk_size=4, num_layers=2,
         hidden=4096, elt=2, kv=2, chunks=1, seed=11),
    # Llama-3-8B GQA shapes scaled down: 8 KV heads x 128, bf16, block 16, chunk 256
    dict(name="gqa_bs16", num_blocks=64, block_size=16, chunk_size=256, num_layers=4,
         hidden=1024, elt=2, kv=2, chunks=3, seed=12),
    # DeepSeek-V2-Lite MLA latent (K only), width 576, bf16, block 64
    dict(name="mla_bs64", num_blocks=32, block_size=64, chunk_size=256, num_layers=3,
         hidden=576, elt=2, kv=1, chunks=2, seed=13),
    # unit of 6 bytes (not a multiple of 4): exercises the narrow-vector path
    dict(name="odd_unit", num_blocks=16, block_size=4, chunk_size=8, num_layers=2,
         hidden=3, elt=2, kv=2, chunks=3, seed=14),
    # TP=8 head shard of Llama-3: one head x 128 x bf16 = 256-byte unit
    dict(name="tp8_shard", num_blocks=128, block_size=16, chunk_size=256, num_layers=5,
         hidden=128, elt=2, kv=2, chunks=4, seed=15),
]


def unit_of(case: dict) -> int:
    return case["hidden"] * case["elt"]


def record_bytes(case: dict) -> int:
    return case["kv"] * case["num_layers"] * case["chunk_size"] * unit_of(case)


def paged_layers(case: dict, seed: int | None = None, zero: bool = False):
    """(k_layers, v_layers or None): per-layer uint8 arrays of
    num_blocks * block_size * unit bytes, K layers first then V layers."""
    n = case["num_blocks"] * case["block_size"] * unit_of(case)
    rng = np.random.default_rng(case["seed"] if seed is None else seed)
    layers = []
    for _ in range(case["kv"] * case["num_layers"]):
        layers.append(np.zeros(n, np.uint8) if zero else rng.integers(0, 256, n, dtype=np.uint8))
    L = case["num_layers"]
    return layers[:L], (layers[L:] if case["kv"] == 2 else None)


def block_ids(case: dict, seed_offset: int = 0) -> np.ndarray:
    """distinct block ids for case['chunks'] chunks, a seeded permutation"""
    bpc = case["chunk_size"] // case["block_size"]
    rng = np.random.default_rng(case["seed"] * 1000 + 7 + seed_offset)
    return rng.permutation(case["num_blocks"])[: bpc * case["chunks"]].astype(np.uint64)


def records_for_scatter(case: dict) -> list[np.ndarray]:
    rng = np.random.default_rng(case["seed"] * 1000 + 99)
    return [rng.integers(0, 256, record_bytes(case), dtype=np.uint8) for _ in range(case["chunks"])]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# block-hash cases: (name, block_size, seed string, token generator spec)
HASH_CASES = [
    ("bs16_small_ids", 16, "0", (0, 256, 5 * 16 + 7)),
    ("bs16_mid_ids", 16, "0", (0, 65536, 6 * 16)),
    ("bs16_llama3_vocab", 16, "0", (0, 128256, 8 * 16 + 3)),
    ("bs16_boundaries", 16, "1234", "boundaries"),
    ("bs64_llama3_vocab", 64, "0", (0, 128256, 4 * 64)),
    ("bs1", 1, "0", (0, 128256, 9)),
    ("bs2", 2, "7", (0, 70000, 10)),
    ("bs3", 3, "7", (0, 70000, 12)),
    ("bs4", 4, "7", (0, 70000, 16)),
    ("bs16_int32_extremes", 16, "42", "extremes"),
    ("bs128_mixed", 128, "3", (0, 300000, 3 * 128)),
]
# the same token specs hashed with vLLM's sha256_cbor (appended after the
# pickle cases so their generator seeds are unchanged)
HASH_CASES_CBOR = [
    ("cbor_bs16_llama3_vocab", 16, "0", (0, 128256, 8 * 16 + 3)),
    ("cbor_bs16_small_ids", 16, "0", (0, 24, 4 * 16)),
    ("cbor_bs16_boundaries", 16, "1234", "boundaries"),
    ("cbor_bs16_int32_extremes", 16, "42", "extremes"),
    ("cbor_bs1", 1, "0", (0, 300, 9)),
    ("cbor_bs3", 3, "7", (0, 70000, 12)),
    ("cbor_bs23", 23, "7", (0, 70000, 46)),
    ("cbor_bs24", 24, "7", (0, 70000, 48)),
    ("cbor_bs64_llama3_vocab", 64, "0", (0, 128256, 4 * 64)),
    ("cbor_bs256", 256, "5", (0, 128256, 2 * 256)),
    ("cbor_bs300", 300, "5", (-1000, 128256, 2 * 300)),
]


def hash_tokens(spec, case_index: int) -> list[int]:
    rng = np.random.default_rng(5000 + case_index)
    if spec == "boundaries":
        base = [0, 1, 254, 255, 256, 257, 65534, 65535, 65536, 65537, 128255, 127, 128, 300, 70000, 5,
                23, 24, 25, 22]
        return base[:16] * 3 + base[4:]
    if spec == "extremes":
        return [-2**31, -1, 2**31 - 1, 0, -256, 256, -65536, 65536,
                -2, 2, 2**31 - 2, -(2**31) + 1, 255, -255, 65535, -65535] * 2
    lo, hi, n = spec
    return rng.integers(lo, hi, n).astype(np.int64).tolist()


# block-hash cases with vLLM's per-block extra keys (hash_block_tokens'
# extra_keys: LoRA name, multimodal (identifier, offset), cache salt, prompt-
# embeds digest): (name, algo, block_size, seed, token spec, extra spec).
# Token generator seeds are 200 + index.
HASH_CASES_EXTRA = [
    ("x_lora_bs16", "sha256", 16, "0", (0, 128256, 4 * 16), "lora"),
    ("x_salt_mm_bs16", "sha256", 16, "0", (0, 128256, 6 * 16 + 5), "salt_mm"),
    ("x_embeds_bs4", "sha256", 4, "3", (0, 70000, 5 * 4), "embeds"),
    ("x_long_bs16", "sha256", 16, "0", (0, 128256, 3 * 16), "long"),
    ("x_mixed_bs1", "sha256", 1, "7", (0, 300, 7), "mixed"),
    ("x_cbor_lora_bs16", "sha256_cbor", 16, "0", (0, 128256, 4 * 16), "lora"),
    ("x_cbor_salt_mm_bs16", "sha256_cbor", 16, "0", (0, 128256, 6 * 16 + 5), "salt_mm"),
    ("x_cbor_long_bs64", "sha256_cbor", 64, "5", (0, 128256, 3 * 64), "long"),
    ("x_cbor_embeds_bs3", "sha256_cbor", 3, "7", (-1000, 70000, 4 * 3), "embeds"),
]


def hash_extra(spec: str, nblocks: int) -> list:
    """per-block extra_keys (a tuple, or None) of an extra spec"""
    if spec == "lora":
        return [("sql-lora-7",)] * nblocks
    if spec == "salt_mm":
        # cache salt on the first block; an image spanning blocks 2-4
        out = []
        for b in range(nblocks):
            keys = []
            if b == 0:
                keys.append("tenant-salt-0001")
            if 2 <= b <= 4:
                keys.append(("6f1c0a93d2e84b57a3c9e0f1b2d4c6a8e0f2b4d6c8a0e2f4b6d8c0a2e4f6b8d0", 16 * (2 - b) + 5))
            out.append(tuple(keys) if keys else None)
        return out
    if spec == "embeds":
        return [(hashlib.sha256(b"prompt-embeds block %d" % b).digest(),) for b in range(nblocks)]
    if spec == "long":
        # segments longer than 256 bytes pass the kernel's ring in pieces
        return [("adapter-" + "x" * (300 + 97 * b), ("mm-" + "ab" * (150 + b), b)) for b in range(nblocks)]
    if spec == "mixed":
        return [None if b % 3 == 0 else ("lora-b", b * 1000 - 7, ("id", -b)) for b in range(nblocks)]
    raise ValueError(spec)
