"""Generate tests/golden/protocol_messages.json from CrossCache's own client
encoder (python/utils/protocol.py, imported by path; it needs only ctypes):

    PYTHONPATH=. python tests/golden/make_protocol_golden.py

Each case records the encoder's inputs and the hex bytes it produced, so the
tests can check this build's encoder (same bytes) and decoder (same fields)
without the reference tree.
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from oracle import reference_root  # noqa: E402

REF = reference_root() / "python" / "utils" / "protocol.py"


def load_ref():
    spec = importlib.util.spec_from_file_location("crosscache_protocol", REF)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    p = load_ref()
    rng = np.random.default_rng(77)
    cases = []

    def key(n):
        return rng.integers(0, 256, n, dtype=np.uint8).tobytes()

    # REGISTER: K and V keys, 72-byte CUDA keys, 3 layers
    lk = [(key(72), key(72)) for _ in range(3)]
    args = dict(node_id=2, uid=7, world_size=4, rank_id=1, num_blocks=16384, block_size=16, element_size=2,
                hidden_dim_size=256, key_len=72, model_name="meta-llama/Meta-Llama-3-8B")
    buf = p.encode_message(p.RequestType.REGISTER_KV_CACHE, args["uid"], p.to_register_payloads(
        args["node_id"], args["world_size"], args["rank_id"], args["num_blocks"], args["block_size"],
        args["element_size"], args["hidden_dim_size"], args["key_len"], args["model_name"], lk))
    cases.append(dict(op="register", args=args, layer_keys=[[k.hex() for k in t] for t in lk],
                      bytes=bytes(buf).hex()))
    # REGISTER: K-only (MLA), 64-byte keys, 1-byte elements
    lk = [(key(64),) for _ in range(2)]
    args = dict(node_id=0, uid=0, world_size=1, rank_id=0, num_blocks=100, block_size=64, element_size=1,
                hidden_dim_size=576, key_len=64, model_name="deepseek-ai/DeepSeek-V2-Lite")
    buf = p.encode_message(p.RequestType.REGISTER_KV_CACHE, args["uid"], p.to_register_payloads(
        args["node_id"], args["world_size"], args["rank_id"], args["num_blocks"], args["block_size"],
        args["element_size"], args["hidden_dim_size"], args["key_len"], args["model_name"], lk))
    cases.append(dict(op="register", args=args, layer_keys=[[k.hex() for k in t] for t in lk],
                      bytes=bytes(buf).hex()))
    # LOOKUP
    keys = [key(32) for _ in range(5)]
    args = dict(node_id=3, uid=123456, world_size=8, model_name="m")
    buf = p.encode_message(p.RequestType.LOOKUP, args["uid"],
                           p.to_lookup_payloads(args["node_id"], keys, args["world_size"], args["model_name"]))
    cases.append(dict(op="lookup", args=args, keys=[k.hex() for k in keys], bytes=bytes(buf).hex()))
    # STORE / LOAD: 2 records of 16 blocks
    for op, rt, mk in (("store", p.RequestType.STORE, p.to_store_payloads),
                       ("load", p.RequestType.LOAD, p.to_load_payloads)):
        keys = [key(32) for _ in range(2)]
        bids = rng.permutation(1 << 20)[:32].tolist()
        args = dict(node_id=5, uid=(1 << 32) - 2 if op == "load" else 9)
        buf = p.encode_message(rt, args["uid"], mk(args["node_id"], keys, bids))
        cases.append(dict(op=op, args=args, keys=[k.hex() for k in keys], block_ids=bids,
                          bytes=bytes(buf).hex()))
    # responses as the server packs them (struct msg_response: uid, ok)
    resp = []
    for uid, st in ((7, 0), (8, 4096), (9, (-2) & 0xFFFFFFFF)):
        r = p.MsgResponse()
        r.uid, r.status = uid, st
        resp.append(dict(uid=uid, status=st, bytes=bytes(r).hex()))
    (HERE / "protocol_messages.json").write_text(json.dumps(dict(requests=cases, responses=resp), indent=1) + "\n")
    print("wrote", HERE / "protocol_messages.json")


if __name__ == "__main__":
    main()
