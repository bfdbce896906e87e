"""Out-of-process deployment on the GPU: a CrossCache server process (CUDA
backend) and a "vLLM worker" process (this one) that registers its paged KV
tensors by 72-byte CUDA IPC keys, stores blocks, asks the scheduler-side
lookup and loads the blocks back into other block ids -- all over ZeroMQ
with the reference's wire protocol."""
import multiprocessing as mp
import os
import time

import pytest

pytestmark = pytest.mark.gpu
zmq = pytest.importorskip("zmq")

NB, BS, H, D, L = 128, 16, 8, 128, 4


def _serve(q, stop):
    import torch

    from demo_b200.server import CacheServer

    torch.cuda.set_device(0)
    try:
        srv = CacheServer("tcp://127.0.0.1:*", 256, 8 * 2 * L * 256 * H * D * 2, None).start()
    except Exception as e:            # report instead of leaving the test waiting
        q.put(("error", repr(e)))
        return
    q.put(("ok", srv.endpoint))
    stop.wait(300)
    srv.stop()


def _kv_layers(layout: str, g):
    """per-layer vLLM KV tensors: FlashAttention [2, NB, BS, H, D], or the
    FlashInfer view [NB, 2, BS, H, D] of head-major blocks (sm_100)"""
    import torch

    if layout == "flash_attn":
        return {f"layer.{i}": torch.randn(2, NB, BS, H, D, generator=g, device="cuda").to(torch.bfloat16)
                for i in range(L)}
    return {f"layer.{i}": torch.randn(NB, 2, H, BS, D, generator=g, device="cuda").to(torch.bfloat16)
            .permute(0, 1, 3, 2, 4) for i in range(L)}


def _blocks(t, layout: str, sl: slice):
    return t[:, sl] if layout == "flash_attn" else t[sl]


@pytest.mark.parametrize("layout", ["flash_attn", "flashinfer_hnd"])
def test_remote_adapters_store_lookup_load(layout):
    """FlashInfer: the REGISTER carries IPC keys of the K and V plane bases
    (V half a block into each layer) and the paged-geometry trailer"""
    import torch

    from demo_b200.adaptor import LoadStoreOp
    from demo_b200.remote import RemoteSchedulerAdapter, RemoteWorkerAdapter

    ctx = mp.get_context("spawn")
    q, stop = ctx.Queue(), ctx.Event()
    p = ctx.Process(target=_serve, args=(q, stop))
    p.start()
    wa = sa = None
    try:
        status, endpoint = q.get(timeout=180)
        assert status == "ok", endpoint
        torch.cuda.set_device(0)
        g = torch.Generator(device="cuda").manual_seed(3)
        layers = _kv_layers(layout, g)
        orig = {k: t.clone() for k, t in layers.items()}
        zctx = zmq.Context.instance()
        wa = RemoteWorkerAdapter(endpoint, zctx, "remote-model", 1, 0, BS, device=0)
        wa.register(layers)
        hashes = [os.urandom(32) for _ in range(32)]          # 2 chunks of 16 blocks
        wa.store_requests(["r1"], [LoadStoreOp(hashes, list(range(32)))])
        assert wa.wait_all(timeout=120) == [0]

        sa = RemoteSchedulerAdapter(endpoint, zctx, "remote-model", 1, 0, BS)
        sa.try_lookup("q", hashes + [os.urandom(32) for _ in range(16)])
        deadline = time.time() + 60
        while (hit := sa.check_lookup_result("q")) is None and time.time() < deadline:
            time.sleep(0.005)
        assert hit == 512

        for t in layers.values():
            _blocks(t, layout, slice(64, 96)).zero_()
        torch.cuda.synchronize()
        wa.load_requests(["r2"], [LoadStoreOp(hashes, list(range(64, 96)))])
        assert wa.wait_all(timeout=120) == [0, 0]
        stores, loads = wa.get_finished(set())
        assert loads == {"r2"}
        torch.cuda.synchronize()
        for k, t in layers.items():
            assert torch.equal(_blocks(t, layout, slice(64, 96)).view(torch.int16),
                               _blocks(orig[k], layout, slice(0, 32)).view(torch.int16)), k
            assert torch.equal(_blocks(t, layout, slice(0, 64)).view(torch.int16),
                               _blocks(orig[k], layout, slice(0, 64)).view(torch.int16)), k
    finally:
        if sa is not None:
            sa.close()
        if wa is not None:
            wa.unregister()
        stop.set()
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert p.exitcode == 0
