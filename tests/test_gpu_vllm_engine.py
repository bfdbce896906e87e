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
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
RECORDS = 16          # 4 prompts of 1024-1135 tokens: 4 whole chunks each


def _run(mode: str, backend: str, kv_dtype: str, model: str = "llama") -> dict:
    pytest.importorskip("vllm")
    p = subprocess.run([sys.executable, os.path.join(HERE, "vllm_engine_run.py"), mode, backend, kv_dtype, model],
                       capture_output=True, text=True, timeout=900, cwd=os.path.dirname(HERE))
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
