"""The connector inside a real vLLM engine (vLLM 0.22, single process): the
first pass stores every whole 256-token chunk of four prompts, the second
pass loads them and must produce the same greedy tokens.  Covers the
FlashInfer backend vLLM picks on sm_100 (head-major blocks, registered
with a block stride and head split), FlashAttention (the reference's dense
layout), an fp8 KV cache, an MLA (K-only latent) model and the layer-wise
mode, where a fully cached prompt must still leave vLLM's scheduler a token
to compute."""
import json
import os
import re
import signal
import socket
import subprocess
import sys
import threading
import time

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
RECORDS = 16          # 4 prompts of 1024-1135 tokens: 4 whole chunks each


def _run(mode: str, backend: str, kv_dtype: str, model: str = "llama", *extra: str) -> dict:
    pytest.importorskip("vllm")
    p = subprocess.run([sys.executable, os.path.join(HERE, "vllm_engine_run.py"), "--mode", mode,
                        "--backend", backend, "--kv-dtype", kv_dtype, "--model", model, *extra],
                       capture_output=True, text=True, timeout=900, cwd=ROOT,
                       env=dict(os.environ, PYTHONPATH=os.pathsep.join(
                           x for x in (ROOT, os.environ.get("PYTHONPATH")) if x)))
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("ENGINE_RESULT ")]
    assert p.returncode == 0 and lines, p.stderr[-4000:]
    return json.loads(lines[-1].split(" ", 1)[1])


@pytest.mark.parametrize("mode,backend,kv_dtype", [("plain", "auto", "auto"), ("layerwise", "auto", "auto"),
                                                   ("plain", "FLASH_ATTN", "auto"), ("plain", "auto", "fp8")])
def test_second_pass_is_served_from_the_cache(mode, backend, kv_dtype):
    """fp8: a 1-byte KV cache (128-byte token units, 64-byte heads)"""
    r = _run(mode, backend, kv_dtype)
    assert r["stored"] == RECORDS and r["loaded_first"] == 0
    assert r["loaded_second"] == RECORDS and r["lookup_hits"] >= RECORDS
    assert r["same_tokens"]
    elt = 1 if kv_dtype == "fp8" else 2
    assert r["element_size"] == elt
    unit = 2 * 64 * elt                     # 2 KV heads of 64
    if backend == "FLASH_ATTN":
        assert (r["block_stride"], r["head_bytes"]) == (0, 0)
    else:                                   # FlashInfer, head-major on sm_100
        assert r["block_stride"] == 2 * 16 * unit and r["head_bytes"] == 64 * elt


@pytest.mark.parametrize("mode", ["plain", "layerwise"])
def test_mla_latent_cache_is_served_from_the_cache(mode):
    """DeepSeek-V2 attention (vLLM picks FLASHINFER_MLA on sm_100): one K-only
    576-wide latent plane per layer, block 64 -- the reference's K-only
    registration, through the real engine"""
    r = _run(mode, "auto", "auto", "mla")
    assert (r["kv"], r["hidden_dim_size"], r["block_size"], r["element_size"]) == (1, 576, 64, 2)
    assert (r["block_stride"], r["head_bytes"]) == (0, 0)
    assert r["stored"] == RECORDS and r["loaded_first"] == 0
    assert r["loaded_second"] == RECORDS and r["same_tokens"]


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("tp", [1, 2])
def test_engine_through_the_server(tp):
    """The engine against one CrossCache server process.  Each rank (with
    TP=2, one vLLM worker process per GPU) registers its KV-head shard by
    CUDA IPC keys; the scheduler's lookups go to the server, where rank 0 of
    the TP group answers, as in the reference; each rank stores and loads
    its own shard records.  The server logs every worker's counters when the
    worker leaves."""
    import torch

    pytest.importorskip("vllm")
    pytest.importorskip("zmq")
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    port = _free_port()
    srv = subprocess.Popen([sys.executable, "-m", "demo_b200.server", "-P", str(port), "--host", "127.0.0.1",
                            "--cachedir", "", "--poolsize", str(1 << 30)],
                           stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, cwd=ROOT,
                           env=dict(os.environ, CROSSCACHE_PYLOG="DEBUG"))
    lines: list[str] = []
    listening = threading.Event()

    def drain():
        for line in srv.stdout:
            lines.append(line)
            if "listening" in line:
                listening.set()
    th = threading.Thread(target=drain, daemon=True)
    th.start()
    try:
        deadline = time.time() + 300
        while not listening.is_set() and srv.poll() is None and time.time() < deadline:
            time.sleep(0.2)
        assert listening.is_set(), "".join(lines)[-4000:]
        r = _run("plain", "auto", "auto", "llama", "--tp", str(tp), "--server-port", str(port))
        assert r["same_tokens"]
    finally:
        srv.send_signal(signal.SIGTERM)
        try:
            srv.wait(timeout=180)
        except subprocess.TimeoutExpired:
            srv.kill()
        th.join(timeout=30)
    assert srv.returncode == 0, "".join(lines)[-4000:]
    per_rank = {}
    for line in lines:
        m = re.search(r"tp=(\d+) rank=(\d+) stats=(\{.*\})", line)
        if m:
            per_rank[int(m.group(2))] = (int(m.group(1)), json.loads(m.group(3)))
    assert sorted(per_rank) == list(range(tp)), "".join(lines)[-4000:]
    requests = [ln.split("server:", 1)[-1].strip() for ln in lines
                if re.search(r"(LOOKUP|Lookup|STORE|LOAD) worker", ln)]
    for rank, (world, st) in per_rank.items():
        assert world == tp
        assert st["stored"] == RECORDS and st["loaded"] == RECORDS, (rank, json.dumps(st), requests[-60:])
