"""ZeroMQ server and wire protocol.

Protocol: this build's encoder reproduces the bytes of CrossCache's own client
encoder (tests/golden/protocol_messages.json, made by
tests/golden/make_protocol_golden.py) and its decoder reads them back.
Server: register / lookup / store / load / unregister through a real ROUTER
socket on the CPU (MEM) backend, with the record bytes checked against the
oracle and the reference's error answers."""
import errno
import json
import logging
import struct
from pathlib import Path

import numpy as np
import pytest

zmq = pytest.importorskip("zmq")

from demo_b200 import protocol as P  # noqa: E402
from demo_b200._lib import CACHE_BACKEND_MEM  # noqa: E402
from demo_b200.mq import MessageQueueClient  # noqa: E402
from demo_b200.server import CacheServer  # noqa: E402
from oracle import kvcopy as ok  # noqa: E402
from tests.golden import gen  # noqa: E402
from tests.test_cache_host import HostKV, keys_for  # noqa: E402

GOLDEN = json.loads((Path(__file__).parent / "golden" / "protocol_messages.json").read_text())


def _reqs(op):
    return [c for c in GOLDEN["requests"] if c["op"] == op]


@pytest.mark.parametrize("case", _reqs("register"), ids=lambda c: c["args"]["model_name"])
def test_register_bytes_equal_reference_encoder(case):
    a = case["args"]
    lk = [tuple(bytes.fromhex(k) for k in t) for t in case["layer_keys"]]
    got = P.encode_register(a["node_id"], a["uid"], a["world_size"], a["rank_id"], a["num_blocks"],
                            a["block_size"], a["element_size"], a["hidden_dim_size"], a["key_len"],
                            a["model_name"], lk)
    assert got.hex() == case["bytes"]
    m = P.decode_request(bytes.fromhex(case["bytes"]))
    assert isinstance(m, P.Register)
    assert (m.node_id, m.uid, m.world_size, m.rank_id, m.num_blocks, m.block_size, m.element_size,
            m.hidden_dim_size, m.key_len, m.model_name) == tuple(a[k] for k in (
                "node_id", "uid", "world_size", "rank_id", "num_blocks", "block_size", "element_size",
                "hidden_dim_size", "key_len", "model_name"))
    assert m.num_layers == len(lk)
    assert m.k_keys == b"".join(t[0] for t in lk)
    assert m.v_keys == (b"".join(t[1] for t in lk) if len(lk[0]) == 2 else None)


def test_lookup_bytes_equal_reference_encoder():
    (case,) = _reqs("lookup")
    a = case["args"]
    keys = [bytes.fromhex(k) for k in case["keys"]]
    got = P.encode_lookup(a["node_id"], a["uid"], keys, a["world_size"], a["model_name"])
    assert got.hex() == case["bytes"]
    m = P.decode_request(got)
    assert isinstance(m, P.Lookup)
    assert (m.keys, m.keys_num, m.key_len, m.world_size, m.model_name) == (
        b"".join(keys), len(keys), 32, a["world_size"], a["model_name"])


@pytest.mark.parametrize("op", ["store", "load"])
def test_transfer_bytes_equal_reference_encoder(op):
    (case,) = _reqs(op)
    a = case["args"]
    keys = [bytes.fromhex(k) for k in case["keys"]]
    code = P.Op.STORE if op == "store" else P.Op.LOAD
    got = P.encode_transfer(code, a["node_id"], a["uid"], keys, case["block_ids"])
    assert got.hex() == case["bytes"]
    m = P.decode_request(got)
    assert isinstance(m, P.Transfer) and m.op == code and m.uid == a["uid"]
    assert m.block_ids.tolist() == case["block_ids"] and m.keys == b"".join(keys)


def test_responses_match_reference_layout():
    for r in GOLDEN["responses"]:
        st = r["status"] - (1 << 32) if r["status"] >= 1 << 31 else r["status"]
        assert P.encode_response(r["uid"], st).hex() == r["bytes"]
        assert P.decode_response(bytes.fromhex(r["bytes"])) == (r["uid"], st)


def test_decoder_rejects_inconsistent_lengths():
    good = P.encode_transfer(P.Op.STORE, 0, 5, [b"a" * 32], list(range(16)))
    with pytest.raises(P.ProtocolError) as e:
        P.decode_request(good[:-1])                       # header len != body
    assert e.value.uid == 5
    bad = bytearray(good)
    struct.pack_into("<I", bad, P.HEADER.size, 1000)      # keys_num past the frame
    with pytest.raises(P.ProtocolError):
        P.decode_request(bytes(bad))
    reg = bytearray(P.encode_register(0, 1, 1, 0, 8, 16, 2, 64, 8, "m", [(b"k" * 8, b"v" * 8)]))
    reg[0] = 0                                            # REGISTER checks the version
    with pytest.raises(P.ProtocolError):
        P.decode_request(bytes(reg))
    with pytest.raises(P.ProtocolError):
        P.decode_request(b"\x01\x09" + bytes(10))         # unknown op
    assert P.decode_request(P.encode_unregister(3, 9)) == P.Unregister(3, 9)


# ---------------------------------------------------------------- server --

CASE = next(c for c in gen.KV_CASES if c["name"] == "gqa_bs16")
BPC = CASE["chunk_size"] // CASE["block_size"]


@pytest.fixture
def server():
    srv = CacheServer("tcp://127.0.0.1:*", CASE["chunk_size"], 20 * gen.record_bytes(CASE), None,
                      CACHE_BACKEND_MEM).start()
    cli = MessageQueueClient(srv.endpoint)
    yield srv, cli
    cli.close()
    srv.stop()


def _register(cli, kv: HostKV, node=0, world=1, rank=0, name="m"):
    """per_len 8: raw pointers, valid because the server runs in this process"""
    k = [struct.pack("<Q", a.ctypes.data) for a in kv.k]
    v = [struct.pack("<Q", a.ctypes.data) for a in kv.v]
    c = kv.case
    return cli.request(lambda uid: P.encode_register(node, uid, world, rank, c["num_blocks"], c["block_size"],
                                                     c["elt"], c["hidden"], 8, name, list(zip(k, v))),
                       timeout=30)


def test_server_store_lookup_load_roundtrip(server, caplog):
    caplog.set_level(logging.INFO, logger="demo_b200.server")
    srv, cli = server
    src, dst = HostKV(CASE), HostKV(CASE, zero=True)
    assert _register(cli, src, node=0) == 0
    assert _register(cli, dst, node=1) == 0          # same (model, tp): shares the pool
    keys = keys_for(CASE["chunks"], seed=21)
    bids, bids2 = gen.block_ids(CASE), gen.block_ids(CASE, seed_offset=1)
    assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys, bids), timeout=30) == 0
    # lookup answers hit tokens (main.c:140), walking from the first key
    assert cli.request(lambda u: P.encode_lookup(0, u, keys, 1, "m"), timeout=30) == CASE["chunks"] * 256
    assert cli.request(lambda u: P.encode_lookup(0, u, [b"\x00" * 32] + keys, 1, "m"), timeout=30) == 0
    assert cli.request(lambda u: P.encode_lookup(0, u, keys, 2, "m"), timeout=30) == 0   # other TP group
    assert cli.request(lambda u: P.encode_transfer(P.Op.LOAD, 1, u, keys, bids2), timeout=30) == 0
    recs = ok.gather(src.k, src.v, bids, CASE["chunk_size"], CASE["block_size"], gen.unit_of(CASE))
    ek, ev = gen.paged_layers(CASE, zero=True)
    ok.scatter(recs, ek, ev, bids2, CASE["chunk_size"], CASE["block_size"], gen.unit_of(CASE))
    assert all(np.array_equal(a, b) for a, b in zip(dst.k, ek))
    assert all(np.array_equal(a, b) for a, b in zip(dst.v, ev))
    assert cli.request(lambda u: P.encode_unregister(1, u), timeout=30) == 0
    assert cli.request(lambda u: P.encode_unregister(0, u), timeout=30) == 0
    # a departing worker's counters are logged (both slots share one entry)
    left = [r.getMessage() for r in caplog.records if "unregistered" in r.getMessage()]
    assert len(left) == 2 and all("model=m tp=1 rank=0" in m for m in left)
    st = json.loads(left[-1].split("stats=", 1)[1])
    assert st["stored"] == CASE["chunks"] and st["loaded"] == CASE["chunks"]


def test_server_error_answers(server):
    srv, cli = server
    kv = HostKV(CASE)
    keys = keys_for(2, seed=22)
    bids = gen.block_ids(CASE)[:2 * BPC]
    # not registered: -EINVAL (main.c:149-153); node id out of range: -ERANGE
    assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys, bids), timeout=30) == -errno.EINVAL
    assert cli.request(lambda u: P.encode_transfer(P.Op.LOAD, 9, u, keys, bids), timeout=30) == -errno.ERANGE
    assert _register(cli, kv, node=9) == -errno.ERANGE
    assert _register(cli, kv, node=0) == 0
    # keys and blocks disagree (the reference aborts on sys_assert)
    assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys, bids[:-1]), timeout=30) == -errno.EINVAL
    # load of keys never stored: -ENOENT
    assert cli.request(lambda u: P.encode_transfer(P.Op.LOAD, 0, u, keys, bids), timeout=30) == -errno.ENOENT
    # a malformed frame still gets an answer for its uid
    assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys, bids)[:-3],
                       timeout=30) == -errno.EINVAL
    # re-register on the same slot replaces the worker
    assert _register(cli, kv, node=0) == 0
    assert cli.request(lambda u: P.encode_transfer(P.Op.STORE, 0, u, keys, bids), timeout=30) == 0
    # unregister of an empty slot is not an error (main.c:113-116)
    assert cli.request(lambda u: P.encode_unregister(5, u), timeout=30) == 0


def test_server_many_concurrent_requests(server):
    """requests from 4 clients interleave on the pools; every answer reaches
    the client and uid that sent it"""
    import threading

    srv, cli = server
    src = HostKV(dict(CASE, num_blocks=256, chunks=16))
    assert _register(cli, src, node=0) == 0
    bids = gen.block_ids(dict(CASE, num_blocks=256, chunks=16))
    errors = []

    def run(t):
        c = MessageQueueClient(srv.endpoint)
        try:
            keys = keys_for(4, seed=100 + t)
            futs = []
            for i in range(20):
                lo = (t * 4 + i % 4) * BPC
                futs.append(c.submit(lambda u, k=keys[i % 4], lo=lo: P.encode_transfer(
                    P.Op.STORE, 0, u, [k], bids[lo:lo + BPC])))
                futs.append(c.submit(lambda u, keys=keys: P.encode_lookup(0, u, keys, 1, "m")))
            res = [f.result(timeout=60) for f in futs]
            assert all(r == 0 for r in res[0::2]), res
            assert all(r % 256 == 0 and 0 <= r <= 4 * 256 for r in res[1::2]), res
            assert c.request(lambda u: P.encode_lookup(0, u, keys, 1, "m"), timeout=30) == 4 * 256
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(repr(e))
        finally:
            c.close()

    ths = [threading.Thread(target=run, args=(t,)) for t in range(4)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    assert not errors, errors
