"""The device block-hash kernel is bit-identical to vLLM's sha256 block hash
(golden vectors from the installed vLLM) and to the oracle restatement."""
import numpy as np
import pytest
import torch

from demo_b200 import hashing
from oracle import blockhash as bh
from tests.golden import gen

pytestmark = pytest.mark.gpu


def test_golden_vectors_host_entry(golden_hashes):
    for case in golden_hashes:
        nh = bytes.fromhex(case["none_hash"])
        extra = ([gen.hash_extra(case["extra"], len(case["tokens"]) // case["block_size"])]
                 if "extra" in case else None)
        got = hashing.block_hashes([case["tokens"]], case["block_size"], nh, algo=case["algo"],
                                   extra_keys=extra)[0]
        assert [h.hex() for h in got] == case["hashes"], case["name"]


@pytest.mark.parametrize("algo", ["sha256", "sha256_cbor"])
def test_random_extra_keys_match_oracle(algo):
    """a batch mixing requests without extra keys, with LoRA / salt / image
    keys, and with segments far longer than the kernel's ring"""
    import hashlib as hl

    rng = np.random.default_rng(77)
    bs = 16
    reqs, extra = [], []
    for r in range(40):
        toks = rng.integers(0, 128256, int(rng.integers(0, 12 * bs))).tolist()
        nb = len(toks) // bs
        kind = r % 4
        if kind == 0:
            ek = None
        elif kind == 1:
            ek = [("lora-%d" % r,)] * nb
        elif kind == 2:
            ek = [(("img-" + hl.sha256(b"%d" % b).hexdigest(), b * 3 - 8),) if b % 2 else None
                  for b in range(nb)]
        else:
            ek = [("s" * int(rng.integers(200, 3000)), hl.sha256(b"e%d" % b).digest(), b) for b in range(nb)]
        reqs.append(toks)
        extra.append(ek)
    nh = bh.none_hash("0", algo)
    got = hashing.block_hashes(reqs, bs, nh, algo=algo, extra_keys=extra)
    exp = bh.batch_block_hashes(reqs, bs, nh, algo, extra)
    assert got == exp


def test_golden_vectors_batched_device_entry(golden_hashes):
    """all golden cases of one block size hashed in one launch, with the
    chains of later cases continued from explicit parents"""
    by_bs = {}
    for c in golden_hashes:
        if "extra" in c:
            continue                       # the host entry covers extra keys
        by_bs.setdefault((c["block_size"], c["none_hash"], c["algo"]), []).append(c)
    for (bs, nh_hex, algo), cases in by_bs.items():
        toks = [c["tokens"] for c in cases]
        lens = [len(t) for t in toks]
        nblk = [n // bs for n in lens]
        flat = torch.tensor([x for t in toks for x in t], dtype=torch.int32, device="cuda")
        toff = torch.tensor(np.cumsum([0] + lens[:-1]), dtype=torch.int64, device="cuda")
        ooff = torch.tensor(np.cumsum([0] + nblk[:-1]), dtype=torch.int64, device="cuda")
        nb = torch.tensor(nblk, dtype=torch.int32, device="cuda")
        out = torch.zeros(sum(nblk), 32, dtype=torch.uint8, device="cuda")
        hashing.block_hashes_device(flat, toff, nb, ooff, bs, bytes.fromhex(nh_hex), out, algo=algo)
        torch.cuda.synchronize()
        got = [bytes(r) for r in out.cpu().numpy()]
        exp = [bytes.fromhex(h) for c in cases for h in c["hashes"]]
        assert got == exp
        # continue each chain from its first hash as an explicit parent
        parents = torch.stack([out[int(o)] for o in ooff.tolist()]).contiguous()
        toff2 = toff + bs
        nb2 = nb - 1
        out2 = torch.zeros_like(out)
        hashing.block_hashes_device(flat, toff2, nb2, ooff, bs, bytes.fromhex(nh_hex), out2, parents=parents,
                                    algo=algo)
        torch.cuda.synchronize()
        for c, o, n in zip(cases, ooff.tolist(), nblk):
            assert [bytes(r).hex() for r in out2[o:o + n - 1].cpu().numpy()] == c["hashes"][1:]


@pytest.mark.parametrize("algo", ["sha256", "sha256_cbor"])
@pytest.mark.parametrize("bs", [16, 64, 300])     # 300: past the pipelined kernel's 256-token limit
def test_random_batch_matches_oracle(bs, algo):
    rng = np.random.default_rng(bs)
    reqs = [rng.integers(-100, 128256, int(rng.integers(0, 40 * bs))).tolist() for _ in range(100)]
    reqs[3] = []                                       # empty request
    reqs[4] = reqs[4][: bs - 1]                        # no full block
    nh = bh.none_hash("0", algo)
    got = hashing.block_hashes(reqs, bs, nh, algo=algo)
    exp = bh.batch_block_hashes(reqs, bs, nh, algo)
    assert got == exp


def test_c2_shape_hash_chain_matches_oracle():
    """configs[1] keys: 64 requests x 2048 tokens U[0,128256) seed 1, block 16"""
    g = torch.Generator().manual_seed(1)
    toks = torch.randint(0, 128256, (64, 2048), generator=g)
    nh = bh.none_hash("0")
    got = hashing.block_hashes(toks.tolist(), 16, nh)
    exp = bh.batch_block_hashes(toks.tolist(), 16, nh)
    assert got == exp
    assert [hashing.chunk_keys(h, 16) for h in got] == [bh.chunk_keys(h, 16) for h in exp]
