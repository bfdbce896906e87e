"""Cross-process registration: a "vLLM worker" process exports 72-byte CUDA
IPC keys of its paged KV layers; a separate "cache server" process imports
them through open_ipc_keys (per_len 72, the reference's register path
src/cache/cache.c:606-619 + npu.cpp:131-180), saves records and loads them
back into the worker's tensors; the worker checks the bytes."""
import ctypes as C
import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NB, BS, H, D, L = 64, 16, 8, 128, 3


def _worker(q_keys, q_done, q_res):
    try:
        _worker_body(q_keys, q_done, q_res)
    except Exception as e:            # unblock the server and the test at once
        q_keys.put(("error", repr(e)))
        q_res.put(("worker-error", repr(e)))
        raise


def _worker_body(q_keys, q_done, q_res):
    import torch

    from demo_b200.ipc import layer_keys

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7)
    # an offset sub-allocation so the 8-byte offset part of the key matters
    pad = torch.empty(4096, dtype=torch.uint8, device="cuda")
    layers = [torch.randn(2, NB, BS, H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(L)]
    orig = [t.clone() for t in layers]
    kk, vk = layer_keys(layers)
    q_keys.put((kk, vk))
    cmd = q_done.get(timeout=120)          # server saved blocks 0..31, cleared them, reloaded at 32..63
    torch.cuda.synchronize()
    ok = all(torch.equal(o[:, :32].view(torch.int16), t[:, 32:].view(torch.int16)) for o, t in zip(orig, layers))
    q_res.put((cmd, ok))
    del pad


def _server(q_keys, q_done, q_res):
    import torch

    from demo_b200 import cache as cc
    from demo_b200._lib import lib

    torch.cuda.set_device(0)
    kk, vk = q_keys.get(timeout=120)
    if kk == "error":
        q_done.put(None)
        q_res.put(("server", 0))
        return
    cc.init(256, 8 * 2 * L * 256 * H * D * 2, None)
    lay = cc.KVLayout(L, NB, BS, H * D, 2, 2)
    w = cc.Worker("ipc-model", lay, [0] * L, [0] * L)
    kb = C.create_string_buffer(kk, len(kk))
    vb = C.create_string_buffer(vk, len(vk))
    w.ctx.per_len = 72
    w.ctx.k_raw_ptrs = C.cast(kb, C.c_void_p)
    w.ctx.v_raw_ptrs = C.cast(vb, C.c_void_p)
    w.register()
    keys = [bytes([i]) * 32 for i in range(2)]
    r1 = w.store(keys, np.arange(32, dtype=np.uint64))
    r2 = w.load(keys, np.arange(32, 64, dtype=np.uint64))
    q_done.put((r1, r2))
    w.unregister()
    cc.exit()
    q_res.put(("server", lib.crosscache_kernel_launches()))


def test_cross_process_ipc_registration():
    ctx = mp.get_context("spawn")
    q_keys, q_done, q_res = ctx.Queue(), ctx.Queue(), ctx.Queue()
    pw = ctx.Process(target=_worker, args=(q_keys, q_done, q_res))
    ps = ctx.Process(target=_server, args=(q_keys, q_done, q_res))
    pw.start()
    ps.start()
    res = [q_res.get(timeout=180) for _ in range(2)]
    pw.join(timeout=60)
    ps.join(timeout=60)
    assert pw.exitcode == 0 and ps.exitcode == 0
    assert not any(r[0] == "worker-error" for r in res), res
    by = {r[0] if r[0] == "server" else "worker": r for r in res}
    assert by["server"][1] > 0
    (r1, r2), ok = by["worker"]
    assert (r1, r2) == (0, 0)
    assert ok
