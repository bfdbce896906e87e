"""One real vLLM engine run with the CrossCache connector, for
tests/test_gpu_vllm_engine.py (run as a child process: vLLM sets up
process-wide state).

A small random-weight model (load_format="dummy", no tokenizer, bf16)
answers four prompts of 1024-1135 token ids twice with greedy sampling and
prefix caching off, so the second pass can only reuse KV through the
connector:
  llama  4 layers, hidden 512, 8 query heads, 2 KV heads of 64, block 16
  mla    DeepSeek-V2 attention, 4 dense layers, hidden 512, 8 heads,
         kv_lora_rank 512 + rope 64 (a 576-wide K-only latent cache), block 64
Prints one JSON line: the registered paged geometry, the worker's stats
after each pass and whether both passes produced the same tokens.

With --server-port the connector talks to a CrossCache server (one process
for all TP ranks, CUDA IPC registration); the counters then live in the
server, which logs them per worker when the worker leaves.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["plain", "layerwise"], default="plain")
    ap.add_argument("--backend", default="auto", help="vLLM attention backend, or auto")
    ap.add_argument("--kv-dtype", default="auto", help="kv_cache_dtype (auto or fp8)")
    ap.add_argument("--model", choices=["llama", "mla"], default="llama")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--server-port", type=int, default=0, help="CrossCache server on 127.0.0.1 (0: in-process)")
    a = ap.parse_args()
    mode, backend, kv_dtype, model = a.mode, a.backend, a.kv_dtype, a.model
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")   # engine in this process
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

    model_dir = tempfile.mkdtemp(prefix=f"crosscache-{model}-")
    if model == "mla":
        from transformers import DeepseekV2Config

        DeepseekV2Config(vocab_size=32000, hidden_size=512, intermediate_size=1024, moe_intermediate_size=256,
                         num_hidden_layers=4, num_attention_heads=8, n_shared_experts=1, n_routed_experts=8,
                         num_experts_per_tok=2, first_k_dense_replace=4, kv_lora_rank=512, q_lora_rank=None,
                         qk_rope_head_dim=64, v_head_dim=128, qk_nope_head_dim=128, max_position_embeddings=4096,
                         architectures=["DeepseekV2ForCausalLM"], torch_dtype="bfloat16").save_pretrained(model_dir)
        block_size = 64
    else:
        from transformers import LlamaConfig

        LlamaConfig(vocab_size=32000, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
                    num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=4096,
                    architectures=["LlamaForCausalLM"], torch_dtype="bfloat16").save_pretrained(model_dir)
        block_size = 16

    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig

    extra = {"cache.pool_size": 1 << 30}
    if mode == "layerwise":
        extra["cache.layerwise"] = True
    if a.server_port:
        extra.update({"cache.server.host": "tcp://127.0.0.1", "cache.server.port": a.server_port})
    kw = {} if backend == "auto" else {"attention_config": {"backend": backend}}
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              enable_prefix_caching=False, gpu_memory_utilization=0.2, max_model_len=2048, block_size=block_size,
              dtype="bfloat16", disable_hybrid_kv_cache_manager=True, seed=0, kv_cache_dtype=kv_dtype,
              tensor_parallel_size=a.tp,
              kv_transfer_config=KVTransferConfig(kv_connector="CrossCacheConnector",
                                                  kv_connector_module_path="demo_b200.connector",
                                                  kv_role="kv_both", kv_connector_extra_config=extra),
              **kw)
    prompts = [{"prompt_token_ids": [(7 * i + 13 * j) % 31000 + 100 for j in range(1024 + 37 * i)]}
               for i in range(4)]
    sp = SamplingParams(max_tokens=16, temperature=0, detokenize=False)
    first = llm.generate(prompts, sp, use_tqdm=False)
    # generate() returns once every request has its tokens; the connector's
    # stores of those requests may still be in flight (vLLM only holds their
    # blocks until the connector reports them done), and a second pass that
    # starts first finds nothing and recomputes.  Let them land.
    chunks = sum(len(p["prompt_token_ids"]) // 256 for p in prompts)
    if a.server_port:
        time.sleep(5.0)           # the counters live in the server process
        second = llm.generate(prompts, sp, use_tqdm=False)
        print("ENGINE_RESULT " + json.dumps({
            "mode": mode, "backend": backend, "model": model, "tp": a.tp, "server": True,
            "same_tokens": all(x.outputs[0].token_ids == y.outputs[0].token_ids for x, y in zip(first, second)),
            "tokens": [list(o.outputs[0].token_ids) for o in second],
        }), flush=True)
        return

    from demo_b200 import connector

    adapter = next(iter(connector._LOCAL_WORKERS.values()))
    deadline = time.time() + 60
    while adapter.worker.stats()["stored"] < chunks and time.time() < deadline:
        time.sleep(0.05)
    st1 = adapter.worker.stats()
    second = llm.generate(prompts, sp, use_tqdm=False)
    st2 = adapter.worker.stats()
    lay = adapter.worker.layout
    print("ENGINE_RESULT " + json.dumps({
        "mode": mode, "backend": backend, "kv_cache_dtype": kv_dtype, "model": model,
        "element_size": lay.element_size, "kv": lay.kv, "block_size": lay.block_size,
        "hidden_dim_size": lay.hidden_dim_size,
        "block_stride": lay.block_stride, "head_bytes": lay.head_bytes,
        "stored": st2["stored"], "loaded_first": st1["loaded"], "loaded_second": st2["loaded"],
        "lookup_hits": st2["lookup_hits"],
        "same_tokens": all(a.outputs[0].token_ids == b.outputs[0].token_ids for a, b in zip(first, second)),
        "tokens": [list(o.outputs[0].token_ids) for o in second],
    }), flush=True)


if __name__ == "__main__":
    main()
