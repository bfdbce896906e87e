"""KV save/load benchmark on the Llama-3-8B GQA workload (32 layers, 8 KV heads
x 128, bf16, block 16, 16384 blocks per layer; 64 requests x 2048 tokens).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One process per GPU (torchrun for N > 1).  At N GPUs the KV heads are split
tensor-parallel (8/N heads per rank); every rank saves and loads its own head
shard (no data exchange) and one NCCL all-reduce(min) per lookup agrees the
per-request hit length before loading.

Printed JSON line (rank 0):
  value      save + load payload GB/s of all ranks through the public C API
             (cache_store / cache_lookup_batch / cache_load) between the paged
             KV cache in HBM and the pinned host record pool, host copies
             inside: each step hashes the token ids on the device, stores
             every request and loads it back, with request r's load (H2D)
             overlapping request r+1's store (D2H) -- the cache serving both
             directions at once.  e2e is the same measurement (with the bytes
             it moves across the host link); `sequential` is the store-all-
             then-load-all step
  link       a synchronised host-link probe (every rank copying at once for
             2 s per direction and both directions together; rank 0 alone at
             N > 1) and the e2e rates as fractions of it
  device     gather + scatter kernels with the records in HBM (CUDA events)
  roofline   the gather kernel that ran (kv_copy_path) vs the measured HBM copy peak
  tp70b / prefix_reuse / mla_evict   the other configurations (Llama-3-70B
             TP at every N; prefix reuse and MLA eviction pressure at N = 1)
  cpu_baseline  the oracle's C restatement of CrossCache's CPU memcpy path
             on the host cores, on a bounded sample of the workload
--impl reference times CrossCache's own CPU transfer path (its mem.cpp
compiled from the reference sources, oracle/_ref) on the host cores, on this
world size's head shard.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KV save/load GB/s per GPU and p50 per-request load latency"
L, KV_HEADS, HEAD_DIM, ELT, BS, NUM_BLOCKS = 32, 8, 128, 2, 16, 16384
REQS, TOKENS, CHUNK, VOCAB = 64, 2048, 256, 128256
GB = 1e9


def duplex_threads(request_bytes: int) -> tuple[int, int]:
    """(save threads, load threads) of the duplex step, from a sweep on B200
    (GB/s of the step, savers x loaders):
                       1x1   1x2   2x2   2x3   4x4
      256 MiB requests 73.8  94.2  82.1  82.1  81.8   (Llama-3-8B, 8 heads)
      2.5 GiB requests 84.8  71.6  92.7  94.9  94.9   (Llama-3-70B, 8 heads)
    With both directions busy, the side with more bytes queued takes the
    link, and short load calls lose ground at every call boundary: one more
    load thread than save threads keeps H2D fed; long requests need two save
    threads to hold D2H's share."""
    saves = 1 if request_bytes < (1 << 30) else 2
    return saves, saves + 1


PRESETS = {
    # the headline config: Llama-3-8B GQA, 64 requests x 2048 tokens
    "llama3-8b": dict(layers=32, requests=64, tokens=2048, blocks=16384, model="llama-3-8b",
                      name="llama3-8b-gqa-kv-offload: 32 layers x 8 KV heads x 128 bf16, block 16, "
                           "16384 blocks/layer; 64 requests x 2048 tokens; 256-token records"),
    # the TP config: Llama-3-70B, 80 layers, heads re-split per world size.
    # 32 x 8192 tokens fill 16384 blocks; 512 more per layer hold request 0's
    # reload while the other requests' blocks are still being saved (the
    # duplex step reloads request r into the blocks request r - 1 was saved
    # from)
    "tp70b": dict(layers=80, requests=32, tokens=8192, blocks=16896, model="llama-3-70b",
                  name="llama3-70b-tp-kv-offload: 80 layers x 8 KV heads x 128 bf16 split over TP ranks, "
                       "block 16, 16896 blocks/layer; 32 requests x 8192 tokens; 256-token records"),
}


def workload_config(tp: int, preset: str = "llama3-8b", **over) -> dict:
    pr = dict(PRESETS[preset], **over)
    paged = 2 * pr["blocks"] * BS * KV_HEADS * HEAD_DIM * ELT * pr["layers"] / tp / 2**30
    recs = 2 * pr["requests"] * pr["tokens"] * KV_HEADS * HEAD_DIM * ELT * pr["layers"] / tp / 2**30
    return {
        "workload": pr["name"],
        "layers": pr["layers"], "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "kv_dtype": "bf16",
        "block_size": BS, "blocks_per_layer": pr["blocks"], "requests": pr["requests"],
        "tokens_per_request": pr["tokens"], "chunk_tokens": CHUNK, "tp": tp,
        "kv_heads_per_rank": KV_HEADS // tp,
        "l2": f"inputs larger than L2: {paged:g} GiB paged cache and {recs:g} GiB of records per rank per step",
    }


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


PATH_NAMES = {1: "kv_copy_kernel (16-byte register copies)",
              2: "kv_copy_bulk_kernel (TMA cp.async.bulk via shared memory)",
              3: "kv_copy_bulk_hnd_kernel (TMA bulk + head-major transpose in shared memory)"}


def profile_for(path: int, unit: int) -> Path:
    """the committed ncu summary of the kernel a launch ran"""
    if path == 1:
        return ROOT / "profiles" / ("kv_copy_register_256b_unit.md" if unit < 1024 else "kv_copy_gather.md")
    return ROOT / "profiles" / ("kv_copy_bulk.md" if path == 2 else "kv_copy_flashinfer_hnd.md")


def ncu_traffic(path: int, unit: int, algorithmic_bytes: int) -> tuple[float | None, str | None]:
    """DRAM bytes of one launch moving `algorithmic_bytes`: the matching ncu
    summary's DRAM bytes per algorithmic byte (a capture larger than L2, so
    traffic grows in proportion), times this launch's algorithmic bytes."""
    f = profile_for(path, unit)
    if not f.exists():
        return None, None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_per_algorithmic_byte:"):
            try:
                return round(float(line.split(":", 1)[1].strip()) * algorithmic_bytes), f"profiles/{f.name}"
            except ValueError:
                return None, None
    return None, None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        mhz, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                mhz.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(mhz)}


def host_info() -> dict:
    """read-only facts about the box the numbers come from"""
    info = {"cpus": os.cpu_count(), "cpu_model": _cpu_model(), "mem_available_gib": round(_mem_available() / 2**30, 1)}
    try:
        q = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id,pcie.link.gen.current,"
                            "pcie.link.width.current,pcie.link.gen.max,pcie.link.width.max",
                            "--format=csv,noheader"], capture_output=True, text=True, timeout=30)
        info["pcie"] = [ln.strip() for ln in q.stdout.splitlines() if ln.strip()]
        t = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, timeout=30)
        # the GPU rows: link type to each peer, CPU and NUMA affinity
        info["topo"] = [" ".join(ln.split()) for ln in t.stdout.splitlines() if ln.startswith("GPU")]
    except Exception as e:
        info["nvidia_smi"] = repr(e)
    return info


def host_copy_gbs(threads: int, seconds: float = 0.5) -> float:
    """Host memory bandwidth as plain copies see it: `threads` threads each
    copy a 64 MiB buffer (numpy releases the GIL) for about `seconds`; read +
    write bytes / s.  Taken before and after the e2e steps, it shows whether
    other jobs on a shared host took memory bandwidth during the run."""
    per = 64 << 20
    src = [np.ones(per, np.uint8) for _ in range(threads)]
    dst = [np.empty(per, np.uint8) for _ in range(threads)]
    with ThreadPoolExecutor(threads) as pool:
        def one_pass():
            list(pool.map(lambda i: np.copyto(dst[i], src[i]), range(threads)))
        one_pass()                                   # touch every page first
        passes, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            one_pass()
            passes += 1
        dt = time.perf_counter() - t0
    return round(2 * threads * per * passes / dt / GB, 2)


def _mem_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    return int(ln.split()[1]) * 1024
    except OSError:
        pass
    return 0


# ---------------------------------------------------------------------------
# CPU legs (oracle port / compiled reference), host memory only

def cpu_sample_run(impl: str, seconds: float | None, iters: int | None, threads: int, shards: int = 1) -> dict:
    """Save then load a bounded sample of the workload through a CPU
    implementation of CrossCache's path: 64 of the 512 full-width records
    (2 GiB per direction), or under a TP split into `shards` the same bytes as
    64 * shards records of one rank's head shard (unit 8/shards heads x 128
    bf16), paged cache in host memory.  Returns GB/s of save+load payload."""
    sys.path.insert(0, str(ROOT))
    from oracle import kvcopy as ok

    chunks = 64 * shards
    nb = chunks * (CHUNK // BS)
    unit = (KV_HEADS // shards) * HEAD_DIM * ELT
    layer_bytes = nb * BS * unit
    k = [np.full(layer_bytes, l, np.uint8) for l in range(L)]
    v = [np.full(layer_bytes, 100 + l, np.uint8) for l in range(L)]
    rec_bytes = 2 * L * CHUNK * unit
    recs = [np.zeros(rec_bytes, np.uint8) for _ in range(chunks)]
    rng = np.random.default_rng(2)
    bids = rng.permutation(nb).astype(np.uint64)
    bids2 = rng.permutation(nb).astype(np.uint64)
    bpc = CHUNK // BS
    payload = 2 * chunks * rec_bytes

    if impl == "reference":
        ref = ok.RefMem()
        slots1 = [ok.slot_mapping(bids[c * bpc:(c + 1) * bpc], BS) for c in range(chunks)]
        slots2 = [ok.slot_mapping(bids2[c * bpc:(c + 1) * bpc], BS) for c in range(chunks)]
        pool = ThreadPoolExecutor(threads)

        def one_step():
            list(pool.map(lambda c: ref.lib.transfer_kvcache(
                ref.ad, C.byref(_params(ref, recs[c], k, v, slots1[c], True, unit))), range(chunks)))
            list(pool.map(lambda c: ref.lib.transfer_kvcache(
                ref.ad, C.byref(_params(ref, recs[c], k, v, slots2[c], False, unit))), range(chunks)))
        # the reference prints a log line per token to stdout: send it to /dev/null
        sys.stdout.flush()
        saved, devnull = os.dup(1), os.open(os.devnull, os.O_WRONLY)
        os.dup2(devnull, 1)
        try:
            times = _time_steps(one_step, seconds, iters)
            ref.libc.fflush(None)
        finally:
            os.dup2(saved, 1)
            os.close(saved)
            os.close(devnull)
        kind, sample = "reference", "CrossCache src/device/mem/mem.cpp TransferKVCache (compiled, oracle/_ref)"
    else:
        def one_step():
            ok.cache_op(recs, k, v, bids, CHUNK, BS, unit, 1, True, threads)
            ok.cache_op(recs, k, v, bids2, CHUNK, BS, unit, 1, False, threads)
        times = _time_steps(one_step, seconds, iters)
        kind, sample = "port", "oracle/kvcopy_oracle.c restatement of mem.cpp:114-173 + cache.c:513-593"
    gbs = [payload / t / GB for t in times]
    shard = (f"{chunks} records of one TP={shards} rank's head shard ({KV_HEADS // shards} heads, {unit}-byte "
             f"units, {rec_bytes >> 20} MiB records; the same bytes as 64 full-width records)"
             if shards > 1 else f"64 of 512 records (1024 blocks, {rec_bytes >> 20} MiB records)")
    return {"value": statistics.median(gbs), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{sample}; {shard}, save then load into a second block table, paged cache in host "
                      f"memory; median of {len(times)} passes",
            "times_s": [round(t, 4) for t in times], "shards": shards, "unit_bytes": unit}


def cpu_geometry_sample(label: str, layers: int, unit: int, block_size: int, kv: int, records: int,
                        threads: int, seconds: float) -> dict:
    """One configuration's CPU baseline: save then load `records` records of
    its geometry (layers, unit bytes, block size, K+V or K only) through the
    oracle's restatement of CrossCache's CPU path (mem.cpp:114-173 under
    cache.c:513-593's chunking), paged cache in host memory, passes repeated
    for about `seconds`.  Returns GB/s of save+load payload (median pass)."""
    from oracle import kvcopy as ok

    nb = records * (CHUNK // block_size)
    layer_bytes = nb * block_size * unit
    k = [np.full(layer_bytes, l, np.uint8) for l in range(layers)]
    v = [np.full(layer_bytes, 100 + l, np.uint8) for l in range(layers)] if kv == 2 else None
    rec_bytes = kv * layers * CHUNK * unit
    recs = [np.zeros(rec_bytes, np.uint8) for _ in range(records)]
    rng = np.random.default_rng(2)
    bids, bids2 = rng.permutation(nb).astype(np.uint64), rng.permutation(nb).astype(np.uint64)

    def one_step():
        ok.cache_op(recs, k, v, bids, CHUNK, block_size, unit, 1, True, threads)
        ok.cache_op(recs, k, v, bids2, CHUNK, block_size, unit, 1, False, threads)
    times = _time_steps(one_step, seconds, None)
    payload = 2 * records * rec_bytes
    return {"value": round(statistics.median(payload / t / GB for t in times), 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{label}: {records} records of {rec_bytes / 2**20:.2f} MiB ({layers} layers, "
                      f"{'K+V' if kv == 2 else 'K only'}, {unit}-byte units, block {block_size}), save then load "
                      f"into a second block table, paged cache in host memory; oracle/kvcopy_oracle.c "
                      f"restatement of mem.cpp:114-173 + cache.c:513-593; median of {len(times)} passes"}


def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _params(ref, rec, k, v, slots, direction, unit):
    from oracle.kvcopy import _RefParams
    kp = np.array([a.ctypes.data for a in k], np.uint64)
    vp = np.array([a.ctypes.data for a in v], np.uint64)
    p = _RefParams(caches=rec.ctypes.data, caches_h=rec.ctypes.data, keys_ptrs=kp.ctypes.data,
                   value_ptrs=vp.ctypes.data, page_buffer_size=0, slot_mapping=slots.ctypes.data,
                   devid=0, caches_element_size=1, num_layers=len(kp), num_tokens=CHUNK,
                   hidden_dim_size=unit, direction=direction)
    p._keep = (kp, vp)
    return p


def _time_steps(fn, seconds, iters):
    times = []
    start = time.perf_counter()
    while True:
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
        if iters is not None and len(times) >= iters:
            break
        if seconds is not None and time.perf_counter() - start >= seconds:
            break
    return times


def run_reference_arm(args) -> None:
    """CrossCache's own CPU path on the host cores, on this world size's work:
    at N GPUs under TP the host serves N head shards, so the sample is made of
    one rank's shard records (unit 8/N heads) holding the same bytes as the
    N = 1 sample, all host threads, one process (rank 0; the others exit)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    shards = max(1, args.gpus)
    have_ref = (ROOT / "oracle" / "_ref" / "libref_mem.so").exists()
    impl = "reference" if have_ref else "port"
    cpu_sample_run(impl, None, args.warmup, threads, shards)      # warm-up passes
    res = cpu_sample_run(impl, None, args.steps, threads, shards)
    v = res["value"]
    line = {"metric": METRIC, "value": round(v, 3), "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(statistics.median(res["times_s"]) * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": workload_config(args.gpus),
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "shard": {"tp": shards, "kv_heads_per_shard": KV_HEADS // shards, "unit_bytes": res["unit_bytes"],
                      "processes": 1, "threads": threads,
                      "note": "the host serves every rank's shard; one process times them on all host threads"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# prefix-reuse and MLA-eviction workloads (1 GPU, through the C API)

def _sha_none(seed: str = "0") -> bytes:
    import hashlib
    import pickle
    return hashlib.sha256(pickle.dumps(seed, protocol=5)).digest()


def _device_hashes(tokens: np.ndarray, lens: np.ndarray, bs: int, dev: int) -> np.ndarray:
    from demo_b200._lib import lib
    nblk = int((lens // bs).sum())
    out = np.zeros((nblk, 32), dtype=np.uint8)
    flat = np.ascontiguousarray(tokens.astype(np.int32))
    n = lib.kv_block_hash_host(dev, flat.ctypes.data, np.ascontiguousarray(lens).ctypes.data, len(lens), bs,
                               _sha_none(), out.ctypes.data)
    assert n == nblk, n
    return out


def run_cache_workload(args) -> None:
    import torch

    from demo_b200 import cache as cc
    from demo_b200._lib import lib
    from oracle.cache_model import LRUPool     # host-side LRU model: the checker only

    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("this workload runs on 1 GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.workload == "prefix-reuse":
        res = _prefix_reuse(dev, cc, lib, args.steps, args.warmup)
    else:
        res = _mla_evict(dev, cc, lib, LRUPool, args.steps, args.warmup)
    print(json.dumps(res), flush=True)


def _prefix_reuse(dev, cc, lib, steps: int, warmup: int, layers=None) -> dict:
    """256 requests = one shared 1024-token prefix + a unique 512-token suffix
    (token ids U[0,128256), seed 1); Llama-3-8B KV shapes (32 layers x 8 KV
    heads x 128 bf16, block 16, 16384 blocks/layer, N(0,1) seed 0).  Per step:
    clear, hash all 256 requests on the device, store the first 128 (block
    table: seeded permutation, seed 2), look up the other 128, load only their
    hit records into a fresh block table (seed 3), one cache_load per request."""
    import torch
    nreq, pre, suf = 256, 1024, 512
    ntok = pre + suf
    if layers is None:
        g = torch.Generator(device=dev).manual_seed(0)
        layers = [torch.randn(2, NUM_BLOCKS, BS, KV_HEADS, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
                  for _ in range(L)]
    layout, kp, vp = cc.layout_from_kv_tensors(layers)
    rb = layout.per_token_size * CHUNK
    gt = torch.Generator().manual_seed(1)
    prefix = torch.randint(0, VOCAB, (pre,), generator=gt)
    toks = torch.cat([prefix.repeat(nreq, 1), torch.randint(0, VOCAB, (nreq, suf), generator=gt)], 1).numpy()
    lens = np.full(nreq, ntok, dtype=np.int64)
    bpc = CHUNK // BS
    kpr = ntok // CHUNK                      # 6 chunk keys per request
    bpr = ntok // BS                         # 96 blocks per request
    save_bt = torch.randperm(NUM_BLOCKS, generator=torch.Generator().manual_seed(2))[: 128 * bpr].numpy().astype(np.uint64)
    load_bt = torch.randperm(NUM_BLOCKS, generator=torch.Generator().manual_seed(3)).numpy().astype(np.uint64)
    uniq = pre // CHUNK + 128 * (kpr - pre // CHUNK)
    cc.init(CHUNK, (uniq + 8) * rb, None)
    w = cc.Worker("llama-3-8b", layout, kp, vp)
    w.register()
    key_nums = np.full(128, kpr, dtype=np.uint32)
    hits = np.zeros(128, dtype=np.uint32)

    src = torch.from_numpy(save_bt[: pre // BS].astype(np.int64)).to(dev)      # request 0's prefix blocks
    snap = [t[:, src].clone() for t in layers]      # what the stored prefix records must hold
    torch.cuda.synchronize()                        # taken before the adaptor's streams touch the cache

    def step(lat, check=False):
        t0 = time.perf_counter()
        w.clear()
        hashes = _device_hashes(toks.reshape(-1), lens, BS, 0)
        keys = np.ascontiguousarray(hashes[bpc - 1::bpc])           # 256 x 6 chunk keys
        kb = keys.tobytes()
        t1 = time.perf_counter()
        assert lib.cache_store(C.byref(w.ctx), kb[: 128 * kpr * 32], 32, save_bt.ctypes.data, 128 * bpr) == 0
        t2 = time.perf_counter()
        kl = kb[128 * kpr * 32:]
        assert lib.cache_lookup_batch(C.byref(w.ctx), kl, key_nums.ctypes.data, 128, 32, hits.ctypes.data) == 0
        off = 0
        for r in range(128):
            h = int(hits[r])
            bt = np.ascontiguousarray(load_bt[off: off + h * bpc])
            ts = time.perf_counter()
            assert lib.cache_load(C.byref(w.ctx), kl[r * kpr * 32: (r * kpr + h) * 32], 32, bt.ctypes.data, h * bpc) == 0
            if lat is not None:
                lat.append(time.perf_counter() - ts)
            off += h * bpc
        t3 = time.perf_counter()
        ok = None
        if check:
            # the load table may overlap the save table (both are drawn from all
            # blocks), so compare every loaded prefix with the pre-step snapshot
            torch.cuda.synchronize()
            ok = True
            for r in range(128):
                dst = torch.from_numpy(load_bt[r * (pre // BS): (r + 1) * (pre // BS)].astype(np.int64)).to(dev)
                ok &= all(torch.equal(sn.view(torch.int16), t[:, dst].view(torch.int16)) for sn, t in zip(snap, layers))
        return t1 - t0, t2 - t1, t3 - t2, int(hits.sum()), ok

    _, _, _, _, ok = step(None, check=True)          # pristine first pass: verified
    for _ in range(max(0, warmup - 1)):
        step(None)
    lat, parts = [], []
    ta = time.perf_counter()
    for _ in range(steps):
        parts.append(step(lat))
    te = time.perf_counter() - ta
    st = w.stats()
    w.unregister()
    cc.exit()
    hit_chunks = parts[-1][3]
    stored_b = uniq * rb
    loaded_b = hit_chunks * rb
    save_s = statistics.median(p[1] for p in parts)
    load_s = statistics.median(p[2] for p in parts)
    return {"metric": METRIC, "value": round((stored_b + loaded_b) * steps / te / GB, 3), "unit": "GB/s",
            "workload": "prefix-reuse: Llama-3-8B KV, 256 requests = shared 1024-token prefix + unique "
                        "512-token suffix; save 128, look up + load the other 128",
            "n_gpus": 1, "steps": steps, "warmup": warmup,
            "ms_per_step": round(te / steps * 1e3, 3), "higher_is_better": True,
            "data": "synthetic", "dtype": "u8",
            "hit_blocks_per_request": hit_chunks * bpc // 128, "hit_rate_chunks": round(hit_chunks / (128 * kpr), 4),
            "records_stored_per_step": uniq, "store_keys_deduplicated_per_step": 128 * kpr - uniq,
            "save_gbs": round(stored_b / save_s / GB, 3), "load_gbs": round(loaded_b / load_s / GB, 3),
            "p50_load_latency_ms": round(statistics.median(lat) * 1e3, 3),
            "hash_store_lookup_load_s": [round(statistics.median(p[i] for p in parts), 4) for i in range(3)],
            "verified_bytes": bool(ok), "stats": st}


def _mla_evict(dev, cc, lib, LRUPool, steps: int, warmup: int) -> dict:
    """DeepSeek-V2-Lite MLA latent cache: 27 layers, K-only width 576 bf16,
    block 64.  512 requests x 4096 tokens = a 2048-token base prefix (one of 64
    seeded bases, chosen Zipf(1.1), seed 4) + a unique 2048-token suffix
    (seed 5).  Host pool = 25 % of the 60.75 GiB working set, so LRU eviction
    runs continuously.  Per request, in order: look up its 16 chunk keys, load
    the hit prefix records into its blocks, write the KV of the missed chunks
    (a pattern derived from each chunk key, standing in for the model), store
    all 16 keys.  Every loaded block is checked against its key's pattern, and
    the hit and eviction counts against the host LRU model."""
    import torch
    nl, width, bs, nreq, ntok, nbase = 27, 576, 64, 512, 4096, 64
    nb = 4096                                         # 64 requests' worth of blocks
    kv = torch.zeros(nl, nb, bs, width, dtype=torch.bfloat16, device=dev)
    layers = [kv[l] for l in range(nl)]
    layout, kp, vp = cc.layout_from_kv_tensors(layers)
    assert layout.kv == 1 and layout.unit == width * 2
    rb = layout.per_token_size * CHUNK                # 7.59 MiB
    bpc = CHUNK // bs                                 # 4 blocks per record
    kpr = ntok // CHUNK                               # 16 chunk keys per request
    total_records = nreq * kpr
    pool_records = total_records // 4                 # 25 % of the working set
    gt = torch.Generator().manual_seed(4)
    bases = torch.randint(0, VOCAB, (nbase, ntok // 2), generator=torch.Generator().manual_seed(6))
    ranks = np.arange(1, nbase + 1, dtype=np.float64)
    pz = ranks ** -1.1
    pz /= pz.sum()
    choice = np.random.default_rng(4).choice(nbase, size=nreq, p=pz)
    suffix = torch.randint(0, VOCAB, (nreq, ntok // 2), generator=torch.Generator().manual_seed(5))
    toks = torch.cat([bases[torch.from_numpy(choice)], suffix], 1).numpy()
    lens = np.full(nreq, ntok, dtype=np.int64)
    hashes = _device_hashes(toks.reshape(-1), lens, bs, 0)
    keys = np.ascontiguousarray(hashes[bpc - 1::bpc]).reshape(nreq, kpr, 32)
    key8 = torch.from_numpy(keys[:, :, :8].copy().view(np.int64).reshape(nreq, kpr)).to(dev)
    lidx = torch.arange(nl, dtype=torch.int64, device=dev).view(nl, 1, 1) << 56
    jidx = (torch.arange(bpc, dtype=torch.int64, device=dev) << 48).view(1, 1, bpc)
    kv64 = kv.view(nl, nb, -1).view(torch.int64)      # [27, nb, 64*576*2/8]
    perm = np.random.default_rng(7).permutation(nb)

    # expected hits / evictions from the host LRU model
    model = LRUPool(pool_records)
    exp_hits = []
    for r in range(nreq):
        kr = [bytes(k) for k in keys[r]]
        h = model.lookup(kr)
        exp_hits.append(h)
        model.store(kr)
    cc.init(CHUNK, pool_records * rb, None)
    w = cc.Worker("deepseek-v2-lite", layout, kp, None)
    w.register()

    def patterns(r, chunks):
        """int64 fill values [27, len(chunks) * 4, 1] of the given chunks of request r"""
        k = key8[r, chunks].view(1, len(chunks), 1)             # [1, c, 1]
        vals = (k ^ lidx) ^ jidx                                # [27, c, 4]
        return vals.reshape(nl, len(chunks) * bpc, 1)

    def one_pass(check: bool):
        w.clear()
        hit_tot, mism, store_s, load_s, lat = 0, 0, 0.0, 0.0, []
        moved_in = moved_out = 0
        for r in range(nreq):
            base = (r % (nb // (kpr * bpc))) * kpr * bpc
            bt = perm[base: base + kpr * bpc].astype(np.uint64)
            kb = keys[r].tobytes()
            h = lib.cache_lookup(C.byref(w.ctx), kb, kpr, 32) // 32
            hit_tot += h
            if h:
                ts = time.perf_counter()
                assert lib.cache_load(C.byref(w.ctx), kb[: h * 32], 32, np.ascontiguousarray(bt[: h * bpc]).ctypes.data,
                                      h * bpc) == 0
                dt = time.perf_counter() - ts
                load_s += dt
                lat.append(dt)
                moved_in += h * rb
                if check:
                    got = kv64[:, torch.from_numpy(bt[: h * bpc].astype(np.int64)).to(dev)]
                    mism += int((got != patterns(r, list(range(h)))).sum())     # every word of every block
            miss = list(range(h, kpr))
            if miss:
                idx = torch.from_numpy(bt[h * bpc:].astype(np.int64)).to(dev)
                kv64[:, idx] = patterns(r, miss).expand(nl, len(miss) * bpc, kv64.shape[2])
            torch.cuda.synchronize()
            before = w.stats()["stored"]
            ts = time.perf_counter()
            assert lib.cache_store(C.byref(w.ctx), kb, 32, np.ascontiguousarray(bt).ctypes.data, kpr * bpc) == 0
            store_s += time.perf_counter() - ts
            moved_out += (w.stats()["stored"] - before) * rb
        return hit_tot, mism, store_s, load_s, lat, moved_in, moved_out

    ev0 = w.stats()["evictions"]
    hit_tot, mism, *_ = one_pass(True)
    ev1 = w.stats()["evictions"]
    for _ in range(max(0, warmup - 1)):
        one_pass(False)
    res = []
    ta = time.perf_counter()
    for _ in range(steps):
        e0 = w.stats()["evictions"]
        res.append(one_pass(False) + (w.stats()["evictions"] - e0,))
    te = time.perf_counter() - ta
    w.unregister()
    cc.exit()
    moved = sum(r[5] + r[6] for r in res)
    lat = [x for r in res for x in r[4]]
    return {"metric": METRIC, "value": round(moved / te / GB, 3), "unit": "GB/s",
            "workload": "mla-evict: DeepSeek-V2-Lite MLA latent (27 layers, 576 bf16, block 64), 512 requests x "
                        "4096 tokens, Zipf(1.1) reuse of 64 base prefixes, host pool 25 % of the working set",
            "n_gpus": 1, "steps": steps, "warmup": warmup,
            "ms_per_step": round(te / steps * 1e3, 3), "higher_is_better": True,
            "data": "synthetic", "dtype": "u8",
            "pool_records": pool_records, "working_set_records": total_records,
            "hit_rate_chunks": round(hit_tot / total_records, 4),
            "evictions_per_pass": ev1 - ev0, "hits_per_pass": hit_tot,
            "lru_model_hits": int(sum(exp_hits)), "lru_model_evictions": model.evictions,
            "hits_match_model": hit_tot == int(sum(exp_hits)), "evictions_match_model": (ev1 - ev0) == model.evictions,
            "save_gbs": round(sum(r[6] for r in res) / sum(r[2] for r in res) / GB, 3),
            "load_gbs": round(sum(r[5] for r in res) / max(1e-9, sum(r[3] for r in res)) / GB, 3),
            "p50_load_latency_ms": round(statistics.median(lat) * 1e3, 3) if lat else None,
            "loaded_block_mismatches": mism, "verified_bytes": mism == 0}


# ---------------------------------------------------------------------------
# optional probes of the headline workload (disk tier, layer-wise, server, paged layouts)

def _fs_type(path: str) -> str:
    best, kind = "", "unknown"
    real = os.path.realpath(path)
    try:
        with open("/proc/mounts") as f:
            for ln in f:
                parts = ln.split()
                if len(parts) > 2 and (real == parts[1] or real.startswith(parts[1].rstrip("/") + "/")) \
                        and len(parts[1]) > len(best):
                    best, kind = parts[1], parts[2]
    except OSError:
        pass
    return kind


def _disk_tier_probe(args, cc, L_, layers, layout, kp, vp, hashes, bt_save, bt_load, disjoint, s) -> dict:
    """Disk tier on a sample of the e2e workload: store the first requests
    with write-behind (store call, then until every file is written), empty
    the memory tier, then load them back from the files (parallel O_DIRECT
    reads + one batched H2D per request).  A fresh directory, removed after."""
    import shutil

    import torch

    n = min(args.disk_requests, s["n_req"])
    keys_per = s["n_tok"] // CHUNK
    nbl = n * s["per_req_blocks"]
    d_payload = n * keys_per * s["rec_bytes"]
    root = os.path.join(args.disk_dir, f"crosscache-bench-{os.getpid()}-{s['rank']}")
    os.makedirs(args.disk_dir, exist_ok=True)
    free_bytes = shutil.disk_usage(args.disk_dir).free
    if free_bytes < 2 * d_payload:
        return {"skipped": f"needs {2 * d_payload} bytes free under the directory, {free_bytes} free"}
    kb = np.ascontiguousarray(hashes[s["bpc"] - 1::s["bpc"]][: n * keys_per]).tobytes()
    save = np.ascontiguousarray(bt_save[:nbl])
    loads = [np.ascontiguousarray(bt_load[r * s["per_req_blocks"]:(r + 1) * s["per_req_blocks"]])
             for r in range(n)]
    b_save = torch.from_numpy(save.astype(np.int64)).to(s["dev"])
    b_load = torch.from_numpy(bt_load[:nbl].astype(np.int64)).to(s["dev"])
    if disjoint:
        for t in layers:
            t[:, b_load] = 0
        torch.cuda.synchronize()         # zeroed before the adaptor's streams write those blocks
    cc.init(CHUNK, (s["nrec"] + 1) * s["rec_bytes"], root)
    try:
        w = cc.Worker("llama-3-8b", layout, kp, vp, node_id=s["local"], world_size=s["world"], rank=s["rank"])
        w.register()
        t0 = time.perf_counter()
        assert L_.cache_store(C.byref(w.ctx), kb, 32, save.ctypes.data, nbl) == 0
        t1 = time.perf_counter()
        w.flush()
        t2 = time.perf_counter()
        w.clear()
        t3 = time.perf_counter()
        for r in range(n):
            kr = kb[r * keys_per * 32:(r + 1) * keys_per * 32]
            assert L_.cache_load(C.byref(w.ctx), kr, 32, loads[r].ctypes.data, s["per_req_blocks"]) == 0
        torch.cuda.synchronize()
        t4 = time.perf_counter()
        ok = all(torch.equal(t[:, b_save].view(torch.int16), t[:, b_load].view(torch.int16)) for t in layers) \
            if disjoint else None
        st = w.stats()
        w.unregister()
    finally:
        cc.exit()
        shutil.rmtree(root, ignore_errors=True)
    return {"records": n * keys_per, "bytes": d_payload, "fs": _fs_type(args.disk_dir),
            "store_call_gbs": round(d_payload / (t1 - t0) / GB, 3),
            "write_gbs": round(d_payload / (t2 - t0) / GB, 3),
            "load_from_files_gbs": round(d_payload / (t4 - t3) / GB, 3),
            "disk_writes": st["disk_writes"], "disk_reads": st["disk_reads"],
            "io_threads": int(os.environ.get("CROSSCACHE_IO_THREADS", "4")),
            "verified_bytes": ok,
            "note": "sample of the e2e workload: store (records in host memory at return, files written "
                    "behind), then every file written; memory emptied; loads read the files"}


def _layerwise_probe(args, cc, layers, layout, kp, vp, hashes, bt_save, bt_load, s) -> dict:
    """A prefix hit served inside the step that computes the request: 4
    requests of 2048 cached tokens (1 GiB of KV) are loaded while a per-layer
    compute proxy for 512 new tokens per request runs (two bf16 GEMMs per
    layer, 2048 x 4096 x 14336 and back: the MLP of Llama-3-8B).  Timed
    (CUDA events, median of the steps): the load alone, the compute alone,
    load then compute, and the layer pipeline (cache_load_async, one launch
    per layer on a side stream, the compute stream waiting on the GPU for
    each layer before its GEMMs)."""
    import torch

    n_req = 4
    prb, bpc = s["per_req_blocks"], s["bpc"]
    keys_per = s["n_tok"] // CHUNK
    kb = [bytes(h) for h in hashes[bpc - 1::bpc][: n_req * keys_per]]
    save = bt_save[: n_req * prb]
    load = bt_load[: n_req * prb]
    dev = s["dev"]
    cc.init(CHUNK, (n_req * keys_per + 1) * s["rec_bytes"], None)
    try:
        w = cc.Worker("llama-3-8b", layout, kp, vp, node_id=s["local"])
        w.register()
        assert w.store(kb, save) == 0
        g = torch.Generator(device=dev).manual_seed(9)
        x = torch.randn(n_req * 512, 4096, generator=g, device=dev).to(torch.bfloat16)
        w1 = (torch.randn(4096, 14336, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        w2 = (torch.randn(14336, 4096, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        L = layout.num_layers
        compute, side = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def forward(h=None):
            y = x
            for l in range(L):
                if h is not None:
                    h.stream_wait(l, compute)
                y = (y @ w1) @ w2
            return y

        def timed(fn):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            with torch.cuda.stream(compute):
                a.record(compute)
                fn()
                b.record(compute)
            torch.cuda.synchronize()
            return a.elapsed_time(b)

        def pipelined():
            h = w.load_async(kb, load)
            ready = torch.cuda.Event()
            ready.record(compute)
            for l in range(L):
                h.layers(l, l + 1, stream=side, wait_event=ready if l == 0 else None)
            forward(h)
            return h

        res = {"load": [], "compute": [], "sequential": [], "pipelined": []}
        for it in range(args.warmup + args.steps):
            t_load = timed(lambda: w.load(kb, load))
            t_comp = timed(forward)
            t_seq = timed(lambda: (w.load(kb, load), forward()))
            hs = []
            t_pipe = timed(lambda: hs.append(pipelined()))
            assert hs[0].finish() == 0
            if it >= args.warmup:
                for k, v in (("load", t_load), ("compute", t_comp), ("sequential", t_seq), ("pipelined", t_pipe)):
                    res[k].append(v)
        ok = all(torch.equal(t[:, torch.from_numpy(save.astype(np.int64)).to(dev)].view(torch.int16),
                             t[:, torch.from_numpy(load.astype(np.int64)).to(dev)].view(torch.int16))
                 for t in layers)
        w.unregister()
    finally:
        cc.exit()
    med = {k: statistics.median(v) for k, v in res.items()}
    hidden = (med["sequential"] - med["pipelined"]) / med["load"] if med["load"] else 0.0
    # 1.0: the shorter of load and compute disappears entirely under the longer
    overlap = (med["load"] + med["compute"] - med["pipelined"]) / min(med["load"], med["compute"])
    return {"requests": n_req, "kv_bytes": n_req * keys_per * s["rec_bytes"],
            "load_ms": round(med["load"], 3), "compute_ms": round(med["compute"], 3),
            "sequential_ms": round(med["sequential"], 3), "pipelined_ms": round(med["pipelined"], 3),
            "load_hidden_frac": round(hidden, 4), "overlap_efficiency": round(overlap, 4),
            "verified_bytes": bool(ok),
            "note": "compute proxy: per layer (2048 x 4096) @ (4096 x 14336) @ (14336 x 4096) bf16; "
                    "load = cache_load (staged, copy engines); pipelined = cache_load_async: per "
                    "layer, copy-engine copies of the layer's slices (one command per run of "
                    "contiguous records) into an HBM ring and a <= 32-CTA scatter, on a side stream"}


def _paged_layout_probe(args, layers, b_save, b_load, s) -> dict:
    """The value step's kernels on vLLM FlashInfer paged layouts: the same KV
    re-laid per layer as [num_blocks][2][heads][block_size][head_dim] (HND,
    what vLLM uses on sm_100) and [num_blocks][2][block_size][heads][head_dim]
    (NHD), registered with block_stride = 2 * block_size * unit (and
    head_bytes for HND).  Per geometry: one gather of every record at the
    save table and one scatter at the load table per step, CUDA events on
    the launch stream; the records must equal the dense layout's gather byte
    for byte and the scatter must reproduce the saved blocks."""
    import torch

    from demo_b200._lib import KVCOPY_FLAG_BULK, KvCopyDesc, lib

    dev, nrec, rec_bytes, bpc = s["dev"], s["nrec"], s["rec_bytes"], s["bpc"]
    n_blocks, unit, n_layers = s["n_blocks"], s["unit"], len(layers)
    hbm_peak, _ = peaks()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ref = torch.empty(nrec * rec_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty_like(ref)
    ptrs = {id(ref): torch.arange(nrec, dtype=torch.int64, device=dev) * rec_bytes + ref.data_ptr(),
            id(out): torch.arange(nrec, dtype=torch.int64, device=dev) * rec_bytes + out.data_ptr()}
    stream = torch.cuda.Stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)

    def desc(kp_d, vp_d, recs, bids, direction, stride=0, head_bytes=0):
        return KvCopyDesc(layer_k=kp_d.data_ptr(), layer_v=vp_d.data_ptr(), records=ptrs[id(recs)].data_ptr(),
                          slots=None, block_ids=bids.data_ptr(), error=err.data_ptr(),
                          page_buffer_size=n_blocks * BS, unit_bytes=unit, num_tokens=CHUNK, block_size=BS,
                          num_layers=n_layers, num_records=nrec, direction=direction, flags=KVCOPY_FLAG_BULK,
                          block_stride=stride, head_bytes=head_bytes)

    dense_k = torch.tensor([t[0].data_ptr() for t in layers], dtype=torch.int64, device=dev)
    dense_v = torch.tensor([t[1].data_ptr() for t in layers], dtype=torch.int64, device=dev)
    with torch.cuda.stream(stream):
        assert lib.kv_copy_launch(C.byref(desc(dense_k, dense_v, ref, b_save, 1)), sptr) == 0
    torch.cuda.synchronize()
    res = {}
    for name, hnd in (("flashinfer_hnd", True), ("flashinfer_nhd", False)):
        fi = [(t.permute(1, 0, 3, 2, 4) if hnd else t.permute(1, 0, 2, 3, 4)).contiguous() for t in layers]
        kp_d = torch.tensor([t.data_ptr() for t in fi], dtype=torch.int64, device=dev)
        vp_d = kp_d + BS * unit
        stride, hb = 2 * BS * unit, (HEAD_DIM * ELT if hnd else 0)
        dg = desc(kp_d, vp_d, out, b_save, 1, stride, hb)
        ds = desc(kp_d, vp_d, out, b_load, 0, stride, hb)
        g_ms, s_ms = [], []
        for it in range(args.warmup + args.steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(stream)
            assert lib.kv_copy_launch(C.byref(dg), sptr) == 0
            ev[1].record(stream)
            assert lib.kv_copy_launch(C.byref(ds), sptr) == 0
            ev[2].record(stream)
            torch.cuda.synchronize()
            if it == 0:
                same_records = bool(torch.equal(out, ref))
            if it >= args.warmup:
                g_ms.append(ev[0].elapsed_time(ev[1]))
                s_ms.append(ev[1].elapsed_time(ev[2]))
        assert int(err.item()) == 0, "kv copy reported an error"
        # with overlapping tables the scatter may overwrite saved blocks: records only
        same_blocks = not s["disjoint"] or all(torch.equal(t[b_save], t[b_load]) for t in fi)
        moved = 2 * nrec * rec_bytes               # read + write bytes of one launch
        gms, sms = statistics.median(g_ms), statistics.median(s_ms)
        res[name] = {"gather_gbs": round(moved / (gms / 1e3) / GB, 1),
                     "scatter_gbs": round(moved / (sms / 1e3) / GB, 1),
                     "gather_frac": round(moved / (gms / 1e3) / GB / hbm_peak, 4),
                     "scatter_frac": round(moved / (sms / 1e3) / GB / hbm_peak, 4),
                     "gather_ms": round(gms, 4), "scatter_ms": round(sms, 4),
                     "path": PATH_NAMES.get(lib.kv_copy_path(C.byref(dg)), "?"),
                     "verified_bytes": bool(same_records and same_blocks)}
        del fi, kp_d, vp_d
        torch.cuda.empty_cache()
    del ref, out
    torch.cuda.empty_cache()
    res["note"] = ("frac of the measured HBM copy peak; same records, block tables and grid as the value step, "
                   "per-layer tensors re-laid in the FlashInfer geometry; records equal the dense layout's")
    return res


def _serve_for_bench(q, stop, pool_bytes):
    import torch

    from demo_b200.server import CacheServer

    torch.cuda.set_device(0)
    try:
        srv = CacheServer("tcp://127.0.0.1:*", CHUNK, pool_bytes, None).start()
    except Exception as e:
        q.put(("error", repr(e)))
        return
    q.put(("ok", srv.endpoint))
    stop.wait(900)
    srv.stop()


def _server_probe(args, layers, hashes, bt_save, bt_load, disjoint, s) -> dict:
    """Save and load of the e2e workload through a server process: the
    worker side (this process) registers its layers by 72-byte CUDA IPC keys
    and sends one STORE and one LOAD message per step carrying every request
    (what the connector's wait_for_save / start_load_kv send), then 64
    single-request LOADs for the per-request latency and 64 LOOKUPs for the
    round trip."""
    import multiprocessing as mp

    import torch
    import zmq

    from demo_b200.adaptor import LoadStoreOp
    from demo_b200.remote import RemoteSchedulerAdapter, RemoteWorkerAdapter

    ctx = mp.get_context("spawn")
    q, stop = ctx.Queue(), ctx.Event()
    p = ctx.Process(target=_serve_for_bench, args=(q, stop, (s["nrec"] + 1) * s["rec_bytes"]))
    p.start()
    wa = sa = None
    try:
        status, endpoint = q.get(timeout=300)
        if status != "ok":
            return {"unavailable": endpoint}
        zctx = zmq.Context.instance()
        wa = RemoteWorkerAdapter(endpoint, zctx, "llama-3-8b", 1, 0, BS, device=s["dev"].index or 0)
        wa.register({f"layer.{i}": t for i, t in enumerate(layers)})
        prb, n_req = s["per_req_blocks"], s["n_req"]
        def ops_for(step: int, table) -> list:
            # fresh keys every step (the first byte carries the step) so each
            # STORE moves every record instead of finding them cached
            hs = [bytes([step & 0xFF]) + bytes(h[1:]) for h in hashes]
            return [LoadStoreOp(hs[r * prb:(r + 1) * prb], table[r * prb:(r + 1) * prb].tolist())
                    for r in range(n_req)]

        ids = [f"r{r}" for r in range(n_req)]
        if disjoint:
            for t in layers:
                t[:, torch.from_numpy(bt_load.astype(np.int64)).to(s["dev"])] = 0
        torch.cuda.synchronize()
        t_st, t_ld = [], []
        for step in range(args.warmup + args.steps):
            save_ops, load_ops = ops_for(step, bt_save), ops_for(step, bt_load)
            t0 = time.perf_counter()
            wa.store_requests(ids, save_ops)
            assert wa.wait_all(timeout=600) == [0]
            t1 = time.perf_counter()
            wa.load_requests(ids, load_ops)
            assert wa.wait_all(timeout=600) == [0, 0]
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            wa.store_futures.clear()
            wa.load_futures.clear()
            if step >= args.warmup:
                t_st.append(t1 - t0)
                t_ld.append(t2 - t1)
        ok = all(torch.equal(t[:, torch.from_numpy(bt_save.astype(np.int64)).to(s["dev"])].view(torch.int16),
                             t[:, torch.from_numpy(bt_load.astype(np.int64)).to(s["dev"])].view(torch.int16))
                 for t in layers) if disjoint else None
        lat = []
        for r in range(n_req):
            t0 = time.perf_counter()
            wa.load_requests([f"l{r}"], [load_ops[r]])
            assert wa.wait_all(timeout=600)[-1] == 0
            lat.append(time.perf_counter() - t0)
            wa.load_futures.clear()
        sa = RemoteSchedulerAdapter(endpoint, zctx, "llama-3-8b", 1, 0, BS)
        rtt, hits = [], 0
        for r in range(n_req):
            t0 = time.perf_counter()
            sa.try_lookup(f"q{r}", save_ops[r].block_hashes)
            h = sa.lookup_futures[f"q{r}"].result(timeout=60)
            rtt.append(time.perf_counter() - t0)
            hits += h
        return {"save_gbs": round(s["payload"] / statistics.median(t_st) / GB, 3),
                "load_gbs": round(s["payload"] / statistics.median(t_ld) / GB, 3),
                "p50_request_load_latency_ms": round(statistics.median(lat) * 1e3, 3),
                "p50_lookup_round_trip_us": round(statistics.median(rtt) * 1e6, 1),
                "lookup_hit_tokens_per_request": hits // n_req, "verified_bytes": ok,
                "note": "server in a second process (CUDA backend, pinned pool there), this process "
                        "registered by 72-byte CUDA IPC keys; one STORE and one LOAD message per step "
                        "carrying all requests, as the connector sends them"}
    finally:
        if sa is not None:
            sa.close()
        if wa is not None:
            wa.unregister()
        stop.set()
        p.join(timeout=300)
        if p.is_alive():
            p.kill()


# ---------------------------------------------------------------------------
# GPU arm

class Ranks:
    """This process's place in the job, and the few collectives the bench
    takes (every rank takes them in the same order)."""

    def __init__(self, world: int, rank: int, local: int, dev, shards: int, shard_index: int):
        self.world, self.rank, self.local, self.dev = world, rank, local, dev
        self.shards, self.shard_index = shards, shard_index

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def _reduce(self, x: float, op) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        import torch.distributed as dist
        return self._reduce(x, dist.ReduceOp.MAX if self.world > 1 else None)

    def min(self, x: float) -> float:
        import torch.distributed as dist
        return self._reduce(x, dist.ReduceOp.MIN if self.world > 1 else None)

    def sum(self, x: float) -> float:
        import torch.distributed as dist
        return self._reduce(x, dist.ReduceOp.SUM if self.world > 1 else None)

    def gather(self, x: float) -> list[float]:
        if self.world == 1:
            return [x]
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        dist.all_gather(out, t)
        return [float(o.item()) for o in out]


def link_probe(rk: Ranks, seconds: float) -> dict:
    """The host link as the e2e steps see it.  After a barrier every rank
    copies 256 MiB pinned <-> device buffers on its own stream (four copies
    in flight) for three windows of `seconds` / 2 each: D2H alone, H2D alone,
    and both directions at once on two streams; at N > 1 also rank 0 alone
    (the others idle), which separates a per-GPU link limit from the box's
    shared one.  Per GPU: bytes / CUDA-event time on the copy stream;
    aggregate: all ranks' bytes / the slowest rank's time; each probe keeps
    its best window."""
    import torch

    mb = 256 << 20
    hd = torch.empty(mb, dtype=torch.uint8, pin_memory=True)      # D2H destination
    hh = torch.empty(mb, dtype=torch.uint8, pin_memory=True)      # H2D source
    dd = torch.zeros(mb, dtype=torch.uint8, device=rk.dev)
    dh = torch.empty(mb, dtype=torch.uint8, device=rk.dev)
    streams = {"d2h": torch.cuda.Stream(rk.dev), "h2d": torch.cuda.Stream(rk.dev)}
    ops = {"d2h": lambda: hd.copy_(dd, non_blocking=True), "h2d": lambda: dh.copy_(hh, non_blocking=True)}

    def run(kinds, secs, active=True):
        torch.cuda.synchronize()
        rk.barrier()
        out = {k: (0.0, 1.0) for k in kinds}
        if active:
            e0 = {k: torch.cuda.Event(enable_timing=True) for k in kinds}
            e1 = {k: torch.cuda.Event(enable_timing=True) for k in kinds}
            ring = {k: [torch.cuda.Event() for _ in range(4)] for k in kinds}
            n = dict.fromkeys(kinds, 0)
            for k in kinds:
                e0[k].record(streams[k])
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < secs:
                for k in kinds:
                    if n[k] >= 4:
                        ring[k][n[k] % 4].synchronize()
                    with torch.cuda.stream(streams[k]):
                        ops[k]()
                    ring[k][n[k] % 4].record(streams[k])
                    n[k] += 1
            for k in kinds:
                e1[k].record(streams[k])
            torch.cuda.synchronize()
            out = {k: (float(n[k] * mb), e0[k].elapsed_time(e1[k]) / 1e3) for k in kinds}
        rk.barrier()
        return out

    def summarise(r, k):
        b, t = rk.gather(r[k][0]), rk.gather(r[k][1])
        rates = sorted(x / y / GB for x, y in zip(b, t))
        return {"per_gpu_min": round(rates[0], 2), "per_gpu_median": round(statistics.median(rates), 2),
                "per_gpu_max": round(rates[-1], 2), "aggregate": round(sum(b) / max(t) / GB, 2)}

    run(["d2h", "h2d"], 0.3)                         # warm the copy paths
    # each probe is WINDOWS synchronized windows; the ceiling is the best
    # window (a host shared with other jobs can dip for a second -- once a
    # 2 s D2H window read 36.6 GB/s on a box whose stores then moved 55.4),
    # and every window's aggregate is reported beside it
    windows = 3
    res = {"seconds_per_window": round(seconds / 2, 3), "windows": windows, "buffer_mib": 256}
    for k in ("d2h", "h2d"):
        ws = [summarise(run([k], seconds / 2), k) for _ in range(windows)]
        res[k] = dict(max(ws, key=lambda w: w["aggregate"]), windows_aggregate=[w["aggregate"] for w in ws])
    best, agg = None, []
    for _ in range(windows):
        r = run(["d2h", "h2d"], seconds / 2)
        w = {k: summarise(r, k) for k in ("d2h", "h2d")}
        w["aggregate"] = round(w["d2h"]["aggregate"] + w["h2d"]["aggregate"], 2)
        agg.append(w["aggregate"])
        if best is None or w["aggregate"] > best["aggregate"]:
            best = w
    res["both"] = dict(best, windows_aggregate=agg)
    if rk.world > 1:
        solo = {}
        for k in ("d2h", "h2d"):
            r = run([k], seconds / 2, active=rk.rank == 0)
            solo[k] = round(r[k][0] / r[k][1] / GB, 2) if rk.rank == 0 else None
        res["solo_rank0"] = solo
    del hd, hh, dd, dh
    torch.cuda.empty_cache()
    return res


def _block_sums(layers, idx, dev) -> list:
    """per (layer, K/V, block) position-weighted int64 checksums of the given blocks"""
    import torch
    out = []
    for t in layers:
        per = []
        for kv in range(2):
            x = t[kv, idx].view(torch.int16).reshape(idx.numel(), -1).to(torch.int64)
            wgt = (torch.arange(x.shape[1], device=dev, dtype=torch.int64) % 251) + 1
            per.append(torch.stack([x.sum(1), (x * wgt).sum(1)]))
            del x
        out.append(torch.stack(per))
    return out


def _sums_equal(a: list, b: list) -> bool:
    import torch
    return all(torch.equal(x, y) for x, y in zip(a, b))


class Offload:
    """One KV-offload workload on this rank's head shard: the seeded paged
    cache (this rank's heads of N(0,1) bf16 values, seed 0), the block tables
    (save: seeded permutation, seed 2; reload: seed 3 over the blocks the save
    did not use when the cache holds both, else over all blocks), the token
    ids (uniform, seed 1) and the keys (vLLM's chained sha256 block hashes,
    one per 256-token record)."""

    def __init__(self, rk: Ranks, preset: str, over: dict | None = None):
        import torch

        from demo_b200 import cache as cc

        pr = dict(PRESETS[preset], **(over or {}))
        self.rk, self.preset, self.model = rk, preset, pr["model"]
        self.n_layers, self.n_req, self.n_blocks, self.n_tok = pr["layers"], pr["requests"], pr["blocks"], pr["tokens"]
        self.full_size = not over
        self.heads = KV_HEADS // rk.shards
        self.unit = self.heads * HEAD_DIM * ELT
        self.bpc = CHUNK // BS
        self.prb = self.n_tok // BS                 # blocks per request
        self.kpr = self.n_tok // CHUNK              # records (keys) per request
        self.nblk = self.n_req * self.prb
        self.nrec = self.nblk // self.bpc
        self.rec_bytes = 2 * self.n_layers * CHUNK * self.unit
        self.payload = self.nrec * self.rec_bytes   # one direction, this rank
        self.group = 1                              # requests per lookup + hit agreement (duplex)
        if self.nblk > self.n_blocks:
            raise SystemExit("blocks per layer must hold the saved blocks")
        dev = rk.dev
        g = torch.Generator(device=dev).manual_seed(0)
        h0 = rk.shard_index * self.heads
        self.layers = []
        for _ in range(self.n_layers):
            full = torch.randn(2, self.n_blocks, BS, KV_HEADS, HEAD_DIM, generator=g, device=dev,
                               dtype=torch.float32).to(torch.bfloat16)
            self.layers.append(full[:, :, :, h0:h0 + self.heads].contiguous())
            del full
        torch.cuda.empty_cache()
        self.layout, self.kp, self.vp = cc.layout_from_kv_tensors(self.layers)
        perm = torch.randperm(self.n_blocks, generator=torch.Generator().manual_seed(2))
        self.bt_save = perm[:self.nblk].numpy().astype(np.uint64)
        self.disjoint = 2 * self.nblk <= self.n_blocks
        spare = perm[self.nblk:]
        free = spare if self.disjoint else perm
        self.reload_perm = free[torch.randperm(free.numel(), generator=torch.Generator().manual_seed(3))
                                ].numpy().astype(np.uint64)
        self.bt_load = self.reload_perm[:self.nblk]
        # rotating reload table: the disjoint reload table, or -- when the
        # cache cannot hold two tables -- request r reloads into the blocks
        # request r - group was saved from (saved before, read by nobody
        # after), the first group into spare blocks.  The duplex step and the
        # batched device step (records reused across batches) need it.
        d = self.group * self.prb
        if self.disjoint:
            self.bt_dup = self.bt_load
        elif spare.numel() >= d:
            self.bt_dup = np.concatenate([spare[:d].numpy().astype(np.uint64), self.bt_save[:self.nblk - d]])
        else:
            self.bt_dup = None
        self.tokens = torch.randint(0, VOCAB, (self.n_req, self.n_tok), generator=torch.Generator().manual_seed(1),
                                    dtype=torch.int64).to(torch.int32).numpy()

    def free(self) -> None:
        import torch
        del self.layers
        torch.cuda.empty_cache()

    def config(self) -> dict:
        if self.full_size:
            return workload_config(self.rk.shards, self.preset)
        c = workload_config(self.rk.shards, self.preset, layers=self.n_layers, requests=self.n_req,
                            blocks=self.n_blocks, tokens=self.n_tok)
        c["workload"] = (f"reduced case for profiling: {self.n_layers} layers, {self.n_req} requests x "
                         f"{self.n_tok} tokens, {self.n_blocks} blocks/layer")
        return c

    # -- kernels only: records in HBM ---------------------------------------
    def device_step(self, steps: int, warmup: int) -> dict:
        """One gather launch (paged -> records) and one scatter launch (records
        -> the reload table) per step, records in HBM (all of them when they
        fit beside the paged cache, else batches reusing one buffer), CUDA
        events on the launch stream."""
        import torch

        from demo_b200._lib import KVCOPY_FLAG_BULK, KvCopyDesc, lib
        rk, dev = self.rk, self.rk.dev
        kp_d = torch.tensor(self.kp, dtype=torch.int64, device=dev)
        vp_d = torch.tensor(self.vp, dtype=torch.int64, device=dev)
        free_b, _ = torch.cuda.mem_get_info(dev)
        batch = int(max(1, min(self.nrec, (free_b - (12 << 30)) // self.rec_bytes)))
        nbatch = (self.nrec + batch - 1) // batch
        records = torch.empty(batch * self.rec_bytes, dtype=torch.uint8, device=dev)
        rec_ptrs = torch.arange(batch, dtype=torch.int64, device=dev) * self.rec_bytes + records.data_ptr()
        b_save = torch.from_numpy(self.bt_save.astype(np.int64)).to(dev)
        # record batches are gathered and scattered in turn, so a scatter must
        # not land on blocks a later batch still gathers: the rotating table
        table = self.bt_dup if self.bt_dup is not None else self.bt_load
        b_load = torch.from_numpy(table.astype(np.int64)).to(dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)

        def desc(bids, first, n, direction):
            return KvCopyDesc(layer_k=kp_d.data_ptr(), layer_v=vp_d.data_ptr(), records=rec_ptrs.data_ptr(),
                              slots=None, block_ids=bids.data_ptr() + first * self.bpc * 8, error=err.data_ptr(),
                              page_buffer_size=self.n_blocks * BS, unit_bytes=self.unit, num_tokens=CHUNK,
                              block_size=BS, num_layers=self.n_layers, num_records=n, direction=direction,
                              flags=KVCOPY_FLAG_BULK)

        batches = [(i * batch, min(batch, self.nrec - i * batch)) for i in range(nbatch)]
        pairs = [(desc(b_save, f, n, 1), desc(b_load, f, n, 0)) for f, n in batches]
        assert sum(lib.kv_copy_payload_bytes(C.byref(g)) for g, _ in pairs) == self.payload
        path = lib.kv_copy_path(C.byref(pairs[0][0]))
        stream = torch.cuda.Stream(dev)
        sptr = C.c_void_p(stream.cuda_stream)

        def step(ev=None):
            for bi, (dg, ds) in enumerate(pairs):
                if ev:
                    ev[bi][0].record(stream)
                assert lib.kv_copy_launch(C.byref(dg), sptr) == 0
                if ev:
                    ev[bi][1].record(stream)
                assert lib.kv_copy_launch(C.byref(ds), sptr) == 0
                if ev:
                    ev[bi][2].record(stream)

        sums0 = _block_sums(self.layers, b_save, dev)
        torch.cuda.synchronize()              # the checksums read blocks the scatter may overwrite
        step()                                # the first step, from the pristine cache: checked
        torch.cuda.synchronize()
        ok = _sums_equal(_block_sums(self.layers, b_load, dev), sums0)
        del sums0
        for _ in range(warmup - 1):
            step()
        torch.cuda.synchronize()
        evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(nbatch)]
               for _ in range(steps)]
        l0 = lib.crosscache_kernel_launches()
        rk.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            step(evs[i])
        t1.record(stream)
        torch.cuda.synchronize()
        rk.barrier()
        launches = lib.crosscache_kernel_launches() - l0
        dt = rk.max(t0.elapsed_time(t1) / 1e3)
        gather_ms = statistics.mean(sum(b[0].elapsed_time(b[1]) for b in e) for e in evs)
        scatter_ms = statistics.mean(sum(b[1].elapsed_time(b[2]) for b in e) for e in evs)
        assert int(err.item()) == 0, "kv copy reported an error"
        if self.disjoint:
            ok = ok and all(torch.equal(t[:, b_save].view(torch.int16), t[:, b_load].view(torch.int16))
                            for t in self.layers)
        ok = bool(rk.min(1.0 if ok else 0.0))
        hbm_peak, peak_kind = peaks()
        alg = 2 * min(batch, self.nrec) * self.rec_bytes        # read + write bytes of one launch
        achieved = 2 * self.payload / (gather_ms / 1e3) / GB
        traffic, traffic_src = ncu_traffic(path, self.unit, alg)
        del records, rec_ptrs
        torch.cuda.empty_cache()
        return {"value": round(rk.sum(2 * self.payload) * steps / dt / GB, 3), "unit": "GB/s",
                "ms_per_step": round(dt / steps * 1e3, 3), "steps": steps, "warmup": warmup,
                "record_batches_per_step": nbatch, "launches": int(launches), "verified_bytes": ok,
                "roofline": {"bound": "hbm", "kernel": PATH_NAMES.get(path, str(path)) + " gather",
                             "path": path, "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                             "traffic": traffic, "traffic_source": traffic_src, "algorithmic_bytes_per_launch": alg,
                             "gather_ms": round(gather_ms, 4), "scatter_ms": round(scatter_ms, 4),
                             "scatter_frac": round(2 * self.payload / (scatter_ms / 1e3) / GB / hbm_peak, 4),
                             "unit_bytes": self.unit},
                "note": "records in HBM; one gather + one scatter per record batch per step; CUDA events on "
                        "the launch stream; frac of the measured HBM copy peak"}

    def hash_kernel(self, steps: int, warmup: int) -> dict:
        """the chained block-hash kernel over every request, tokens in HBM"""
        import torch

        from demo_b200.hashing import block_hashes_device
        dev = self.rk.dev
        nh = _sha_none()
        tok_d = torch.from_numpy(self.tokens.reshape(-1).copy()).to(dev)
        toff_d = torch.arange(self.n_req, dtype=torch.int64, device=dev) * self.n_tok
        ooff_d = torch.arange(self.n_req, dtype=torch.int64, device=dev) * self.prb
        nb_d = torch.full((self.n_req,), self.prb, dtype=torch.int32, device=dev)
        hout = torch.empty(self.nblk, 32, dtype=torch.uint8, device=dev)
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                block_hashes_device(tok_d, toff_d, nb_d, ooff_d, BS, nh, hout, stream=stream)
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            h0.record(stream)
            for _ in range(steps):
                block_hashes_device(tok_d, toff_d, nb_d, ooff_d, BS, nh, hout, stream=stream)
            h1.record(stream)
        torch.cuda.synchronize()
        ms = h0.elapsed_time(h1) / steps
        return {"kernel_ms": round(ms, 4), "blocks": self.nblk, "chains": self.n_req,
                "blocks_per_s": round(self.nblk / (ms / 1e3), 1),
                "sha256_compressions_per_s": round(3 * self.nblk / (ms / 1e3), 1),
                "us_per_block_along_a_chain": round(ms * 1e3 / self.prb, 3),
                "bound": "integer latency along each chain (3 SHA-256 compressions per 16-token block)"}

    # -- end to end: the public C API, pinned host record pool ----------------
    def _fit(self, pool_budget: float, batches: int, limit: int) -> int:
        """requests per batch whose records (`batches` batches of them) fit in
        this rank's share of free host memory, agreed over the ranks"""
        fit = int(pool_budget // self.rec_bytes) - 1
        return int(self.rk.min(min(limit, max(0, fit) // (batches * self.kpr))))

    def e2e(self, steps: int, warmup: int, pool_budget: float, threads: tuple | None = None) -> dict:
        """Two end-to-end steps through cache_store / cache_lookup_batch /
        cache_load (host clock, every H2D / D2H inside).

        sequential: hash the batch's token ids on the device, store every
          request, look the keys up, agree the hit lengths over the ranks
          (all-reduce(min)), load every request back into the reload table.
        duplex: the serving pattern -- step k hashes batch k (fresh prompts:
          the NONE_HASH seed is the step number), agrees the hit lengths of
          batch k-1 (saved in the previous step) in one all-reduce, then
          stores batch k on one thread while loading batch k-1 on another, so
          D2H and H2D run at once and no collective sits between them.  The
          pool holds three batches, so LRU eviction always takes the batch
          loaded two steps before.  Stores read the save table while loads
          write the disjoint reload table (a cache too small for two tables
          runs fewer requests per step, said in `requests_per_step`).

        Pools are sized to the records each step keeps (fewer requests per
        step when this rank's share of free host memory cannot hold them)."""
        import torch

        from demo_b200 import cache as cc
        from demo_b200._lib import lib
        from demo_b200.tp import agree_min_hits

        rk, dev = self.rk, self.rk.dev
        kpr, prb, bpc = self.kpr, self.prb, self.bpc
        out = {"requests": self.n_req, "steps": steps, "warmup": warmup}

        def timed(fn, state):
            lat: list[float] = []
            parts = []
            l0 = lib.crosscache_kernel_launches()
            rk.barrier()
            torch.cuda.synchronize()
            ts0 = time.perf_counter()
            for _ in range(steps):
                parts.append(fn(state, lat))
            torch.cuda.synchronize()
            te = rk.max(time.perf_counter() - ts0)
            rk.barrier()
            return parts, lat, te, lib.crosscache_kernel_launches() - l0

        def med(parts, key):
            return rk.max(statistics.median(p[key] for p in parts))

        def lat_stats(lat):
            return (round(rk.max(statistics.median(lat)) * 1e3, 3),
                    round(rk.max(float(np.percentile(lat, 90))) * 1e3, 3))

        def hasher(R):
            flat = np.ascontiguousarray(self.tokens[:R].reshape(-1))
            lens = np.full(R, self.n_tok, dtype=np.int64)
            hashes = np.zeros((R * prb, 32), dtype=np.uint8)

            def keys(seed: str) -> bytes:
                n = lib.kv_block_hash_host(rk.local, flat.ctypes.data, lens.ctypes.data, R, BS, _sha_none(seed),
                                           hashes.ctypes.data)
                assert n == R * prb, n
                return np.ascontiguousarray(hashes[bpc - 1::bpc]).tobytes()
            return keys, flat.nbytes + lens.nbytes, hashes.nbytes

        def worker(nrec):
            cc.init(CHUNK, (nrec + 1) * self.rec_bytes, None)
            w = cc.Worker(self.model, self.layout, self.kp, self.vp, node_id=rk.local, world_size=rk.world,
                          rank=rk.rank)
            w.register()
            return w

        def ok_all(x: bool) -> bool:
            return bool(rk.min(1.0 if x else 0.0))

        # ---------------- sequential ----------------
        R = self._fit(pool_budget, 1, self.n_req)
        if R < 1:
            out["sequential"] = {"skipped": f"one request's records do not fit in {pool_budget / 2**30:.1f} GiB"}
        else:
            nblk, payload = R * prb, R * kpr * self.rec_bytes
            keys, up_b, down_b = hasher(R)
            key_nums = np.full(R, kpr, dtype=np.uint32)
            hits = np.zeros(R, dtype=np.uint32)
            save_all = np.ascontiguousarray(self.bt_save[:nblk])
            loads = [np.ascontiguousarray(self.bt_load[r * prb:(r + 1) * prb]) for r in range(R)]
            b_save = torch.from_numpy(save_all.astype(np.int64)).to(dev)
            b_load = torch.from_numpy(self.bt_load[:nblk].astype(np.int64)).to(dev)
            w = worker(R * kpr)

            def seq_step(state, lat):
                t0 = time.perf_counter()
                w.clear()
                kb = keys("0")
                th = time.perf_counter()
                rk.barrier()                         # every rank starts its stores together
                t1 = time.perf_counter()
                ret = lib.cache_store(C.byref(w.ctx), kb, 32, save_all.ctypes.data, nblk)
                assert ret == 0, ret
                t2 = time.perf_counter()
                rk.barrier()                         # the ranks' save skew, kept out of the agreement
                t3 = time.perf_counter()
                assert lib.cache_lookup_batch(C.byref(w.ctx), kb, key_nums.ctypes.data, R, 32,
                                              hits.ctypes.data) == 0
                hit = agree_min_hits(hits, device=dev)       # NCCL all-reduce(min) under TP
                t4 = time.perf_counter()
                for r in range(R):
                    h = int(hit[r])
                    ts = time.perf_counter()
                    ret = lib.cache_load(C.byref(w.ctx), kb[r * kpr * 32:(r * kpr + h) * 32], 32,
                                         loads[r].ctypes.data, h * bpc)
                    assert ret == 0, ret
                    if lat is not None:
                        lat.append(time.perf_counter() - ts)
                t5 = time.perf_counter()
                return dict(hash=th - t0, store=t2 - t1, skew=t3 - t2, agree=t4 - t3, load=t5 - t4, total=t5 - t0,
                            hits=int(hit.sum()))

            try:
                if self.disjoint:
                    for t in self.layers:    # the exact final check needs the destination blocks empty
                        t[:, b_load] = 0
                sums = _block_sums(self.layers, b_save, dev)
                torch.cuda.synchronize()     # zeroing and checksums done before the adaptor's streams copy
                seq_step(None, None)         # checked first step
                torch.cuda.synchronize()
                ok = _sums_equal(_block_sums(self.layers, b_load, dev), sums)
                del sums
                for _ in range(warmup - 1):
                    seq_step(None, None)
                parts, lat, te, launches = timed(seq_step, None)
                if self.disjoint:
                    ok = ok and all(torch.equal(t[:, b_save].view(torch.int16), t[:, b_load].view(torch.int16))
                                    for t in self.layers)
                ok = ok_all(ok)
                evictions = w.stats()["evictions"]
            finally:
                w.unregister()
                cc.exit()
            p50, p90 = lat_stats(lat)
            out["sequential"] = {
                "value": round(rk.sum(2 * payload) * steps / te / GB, 3), "unit": "GB/s",
                "ms_per_step": round(te / steps * 1e3, 3), "requests_per_step": R,
                "save_gbs_aggregate": round(rk.sum(payload) / med(parts, "store") / GB, 3),
                "load_gbs_aggregate": round(rk.sum(payload) / med(parts, "load") / GB, 3),
                "save_gbs_per_gpu_slowest": round(payload / med(parts, "store") / GB, 3),
                "load_gbs_per_gpu_slowest": round(payload / med(parts, "load") / GB, 3),
                "hash_ms": round(med(parts, "hash") * 1e3, 3),
                "save_skew_ms": round(med(parts, "skew") * 1e3, 3),
                "lookup_agree_ms": round(med(parts, "agree") * 1e3, 3),
                "p50_load_latency_ms": p50, "p90_load_latency_ms": p90,
                "hit_blocks_per_request": parts[-1]["hits"] * bpc // R, "gpu_launches": int(launches),
                "h2d_bytes_per_step": int(payload + up_b + 2 * nblk * 8), "d2h_bytes_per_step": int(payload + down_b),
                "evictions": evictions, "verified_bytes": ok,
                "note": "hash; barrier; cache_store of every request; barrier (save skew); "
                        "cache_lookup_batch + all-reduce(min); one cache_load per request"}

        # ---------------- duplex ----------------
        limit = self.n_req if self.disjoint else self.n_blocks // (2 * prb)
        R = self._fit(pool_budget, 3, limit)
        if R < 1:
            out["duplex"] = None
            return out
        nblk, payload = R * prb, R * kpr * self.rec_bytes
        keys, up_b, down_b = hasher(R)
        key_nums = np.full(R, kpr, dtype=np.uint32)
        hits = np.zeros(R, dtype=np.uint32)
        # a cache that cannot hold the save and reload tables of every request
        # runs fewer requests: their reload table is the seeded reload
        # permutation without the blocks those requests are saved from
        rest = self.reload_perm if self.disjoint else self.reload_perm[
            ~np.isin(self.reload_perm, self.bt_save[:nblk])]
        dl_table = np.ascontiguousarray(rest[:nblk])
        n_save, n_load = threads or duplex_threads(kpr * self.rec_bytes)
        saves = [np.ascontiguousarray(self.bt_save[r * prb:(r + 1) * prb]) for r in range(R)]
        dloads = [np.ascontiguousarray(dl_table[r * prb:(r + 1) * prb]) for r in range(R)]
        b_save = torch.from_numpy(self.bt_save[:nblk].astype(np.int64)).to(dev)
        b_dl = torch.from_numpy(dl_table.astype(np.int64)).to(dev)
        w = worker(3 * R * kpr)

        def duplex_step(state, lat):
            k = state["k"] + 1
            t0 = time.perf_counter()
            kb, kprev = keys(str(k)), state["prev"]
            th = time.perf_counter()
            rk.barrier()
            t1 = time.perf_counter()
            assert lib.cache_lookup_batch(C.byref(w.ctx), kprev, key_nums.ctypes.data, R, 32, hits.ctypes.data) == 0
            hit = agree_min_hits(hits, device=dev)           # one all-reduce(min) for the step's loads
            t2 = time.perf_counter()
            errs: list = []

            def saver(j):
                for r in range(j, R, n_save):
                    ret = lib.cache_store(C.byref(w.ctx), kb[r * kpr * 32:(r + 1) * kpr * 32], 32,
                                          saves[r].ctypes.data, prb)
                    if ret:
                        errs.append(("store", r, ret))

            load_end = [0.0] * n_load

            def loader(j):
                for r in range(j, R, n_load):
                    h = int(hit[r])
                    ts = time.perf_counter()
                    ret = lib.cache_load(C.byref(w.ctx), kprev[r * kpr * 32:(r * kpr + h) * 32], 32,
                                         dloads[r].ctypes.data, h * bpc)
                    if ret:
                        errs.append(("load", r, ret))
                    if lat is not None:
                        lat.append(time.perf_counter() - ts)
                load_end[j] = time.perf_counter()

            ths = [threading.Thread(target=saver, args=(j,), daemon=True) for j in range(n_save)] + [
                threading.Thread(target=loader, args=(j,), daemon=True) for j in range(n_load)]
            for t in ths:
                t.start()
            for t in ths:
                t.join()
            t_l = max(load_end)
            t3 = time.perf_counter()
            assert not errs, errs
            state.update(k=k, prev=kb)
            return dict(hash=th - t0, skew=t1 - th, agree=t2 - t1, load=t_l - t2, io=t3 - t2, total=t3 - t0,
                        hits=int(hit.sum()))

        try:
            w.clear()
            kb0 = keys("0")                      # batch 0, stored before the first step
            assert lib.cache_store(C.byref(w.ctx), kb0, 32, np.ascontiguousarray(self.bt_save[:nblk]).ctypes.data,
                                   nblk) == 0
            state = {"k": 0, "prev": kb0}
            for t in self.layers:                # the reload blocks start empty: every byte is checked
                t[:, b_dl] = 0
            sums = _block_sums(self.layers, b_save, dev)
            torch.cuda.synchronize()             # zeroing and checksums done before the adaptor's streams copy
            duplex_step(state, None)             # checked first step: loads batch 0
            torch.cuda.synchronize()
            ok = _sums_equal(_block_sums(self.layers, b_dl, dev), sums)
            del sums
            for _ in range(warmup - 1):
                duplex_step(state, None)
            parts, lat, te, launches = timed(duplex_step, state)
            ok = ok and all(torch.equal(t[:, b_save].view(torch.int16), t[:, b_dl].view(torch.int16))
                            for t in self.layers)
            ok = ok_all(ok)
            st = w.stats()
        finally:
            w.unregister()
            cc.exit()
        p50, p90 = lat_stats(lat)
        out["duplex"] = {
            "value": round(rk.sum(2 * payload) * steps / te / GB, 3), "unit": "GB/s",
            "ms_per_step": round(te / steps * 1e3, 3), "requests_per_step": R,
            "pool_bytes_per_rank": (3 * R * kpr + 1) * self.rec_bytes,
            "hash_ms": round(med(parts, "hash") * 1e3, 3),
            "step_skew_ms": round(med(parts, "skew") * 1e3, 3),
            "lookup_agree_ms": round(med(parts, "agree") * 1e3, 3),
            "load_phase_ms": round(med(parts, "load") * 1e3, 3),
            "store_and_load_ms": round(med(parts, "io") * 1e3, 3),
            "p50_load_latency_ms": p50, "p90_load_latency_ms": p90,
            "hit_blocks_per_request": parts[-1]["hits"] * bpc // R, "gpu_launches": int(launches),
            "h2d_bytes_per_step": int(payload + up_b + 2 * nblk * 8), "d2h_bytes_per_step": int(payload + down_b),
            "evictions": st["evictions"], "verified_bytes": ok,
            "save_threads": n_save, "load_threads": n_load,
            "note": ("per step: hash batch k (fresh prompts: the NONE_HASH seed is the step number); barrier "
                     "(step skew); cache_lookup_batch + one all-reduce(min) over batch k-1's keys; then "
                     f"cache_store of batch k ({n_save} thread(s), one call per request) while cache_load "
                     f"brings batch k-1 back ({n_load} threads, one call per request): D2H and H2D at once, "
                     "no collective between them; the load latency is with the other loads and saves in "
                     "flight. Pool of three batches: LRU evicts the batch loaded two steps before.")}
        return out

    # -- the no-allocation entry point on the same shapes ---------------------
    def noalloc_step(self, steps: int, warmup: int) -> dict:
        """kv_copy_noalloc (host arrays, static scratch) with KVCOPY_FLAG_BULK:
        one gather + one scatter of every record per step, records in HBM,
        CUDA events around each call on the stream it is given; the records
        must equal kv_copy_launch's and the scatter must reproduce the saved
        blocks"""
        import torch

        from demo_b200._lib import KVCOPY_FLAG_BULK, lib
        dev = self.rk.dev
        records = torch.empty(self.nrec * self.rec_bytes, dtype=torch.uint8, device=dev)
        rp = (np.arange(self.nrec, dtype=np.uint64) * np.uint64(self.rec_bytes)) + np.uint64(records.data_ptr())
        kp, vp = np.asarray(self.kp, np.uint64), np.asarray(self.vp, np.uint64)
        bs_, bl_ = np.ascontiguousarray(self.bt_save), np.ascontiguousarray(self.bt_load)
        stream = torch.cuda.Stream(dev)

        def call(bids, direction):
            return lib.kv_copy_noalloc(self.rk.local, kp.ctypes.data, vp.ctypes.data, rp.ctypes.data,
                                       bids.ctypes.data, self.nrec, self.n_blocks * BS, self.unit, CHUNK, BS,
                                       self.n_layers, direction, KVCOPY_FLAG_BULK, C.c_void_p(stream.cuda_stream))

        assert call(bs_, 1) == 0 and call(bl_, 0) == 0
        ok = all(torch.equal(t[:, torch.from_numpy(bs_.astype(np.int64)).to(dev)].view(torch.int16),
                             t[:, torch.from_numpy(bl_.astype(np.int64)).to(dev)].view(torch.int16))
                 for t in self.layers) if self.disjoint else None
        g_ms, s_ms = [], []
        for it in range(warmup + steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(stream)
            assert call(bs_, 1) == 0
            ev[1].record(stream)
            assert call(bl_, 0) == 0
            ev[2].record(stream)
            torch.cuda.synchronize()
            if it >= warmup:
                g_ms.append(ev[0].elapsed_time(ev[1]))
                s_ms.append(ev[1].elapsed_time(ev[2]))
        hbm_peak, _ = peaks()
        moved = 2 * self.payload
        gms, sms = statistics.median(g_ms), statistics.median(s_ms)
        del records
        torch.cuda.empty_cache()
        return {"gather_gbs": round(moved / (gms / 1e3) / GB, 1), "scatter_gbs": round(moved / (sms / 1e3) / GB, 1),
                "gather_frac": round(moved / (gms / 1e3) / GB / hbm_peak, 4),
                "scatter_frac": round(moved / (sms / 1e3) / GB / hbm_peak, 4),
                "gather_ms": round(gms, 4), "scatter_ms": round(sms, 4), "records": self.nrec,
                "block_ids": self.nblk, "flags": "KVCOPY_FLAG_BULK", "steps": steps, "warmup": warmup,
                "verified_bytes": ok,
                "note": "each call uploads its host arrays into the static scratch, launches, and waits on the "
                        "host; the time includes the uploads and the wait"}


def _sub_line(res: dict, keep: tuple) -> dict:
    return {k: res[k] for k in keep if k in res}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--link-seconds", type=float, default=2.0, help="seconds per host-link probe")
    ap.add_argument("--skip-e2e", action="store_true", help="kernels only (for ncu captures)")
    ap.add_argument("--no-subs", action="store_true", help="skip the tp70b / prefix-reuse / mla-evict objects")
    ap.add_argument("--duplex-threads", default=None,
                    help="SAVE,LOAD thread counts of the duplex step (default: duplex_threads())")
    ap.add_argument("--sub-steps", type=int, default=3, help="timed steps of each sub-workload")
    ap.add_argument("--sub-warmup", type=int, default=2, help="warm-up steps of each sub-workload (the first checked)")
    ap.add_argument("--disk-dir", default=None,
                    help="also time the disk tier in a fresh directory under this path (off by default)")
    ap.add_argument("--disk-requests", type=int, default=8, help="requests of the disk-tier sample")
    ap.add_argument("--layerwise", action="store_true",
                    help="also time a layer-pipelined load against a per-layer compute proxy")
    ap.add_argument("--via-server", action="store_true",
                    help="also time save/load through a CrossCache server process (ZeroMQ + CUDA IPC)")
    ap.add_argument("--layers", type=int, default=None, help="smaller cases for ncu captures only")
    ap.add_argument("--requests", type=int, default=None)
    ap.add_argument("--blocks-per-layer", type=int, default=None)
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--emulate-tp", type=int, default=1,
                    help="1 process: rank 0's head shard of a TP split (ncu captures of shard kernels only)")
    ap.add_argument("--workload", default="llama3-8b",
                    choices=["llama3-8b", "tp70b", "prefix-reuse", "mla-evict"],
                    help="llama3-8b: the headline save/load config; tp70b: the Llama-3-70B TP "
                         "config; prefix-reuse and mla-evict: the prefix-reuse and MLA-eviction "
                         "configs (1 GPU)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.workload in ("prefix-reuse", "mla-evict"):
        run_cache_workload(args)
        return

    import torch
    import torch.distributed as dist

    from demo_b200 import cache as cc
    from demo_b200._lib import lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    if world > 1 and args.emulate_tp != 1:
        raise SystemExit("--emulate-tp is for one process")
    shards = world if world > 1 else args.emulate_tp
    if KV_HEADS % shards:
        raise SystemExit("the TP size must divide 8 KV heads")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    rk = Ranks(world, rank, local, dev, shards, rank if world > 1 else 0)
    # this rank's share of the host memory free at start (ranks share the host)
    budget = rk.min(0.6 * _mem_available() / world)
    hinfo = host_info() if rank == 0 else None
    over = {k: v for k, v in (("layers", args.layers), ("requests", args.requests),
                               ("blocks", args.blocks_per_layer), ("tokens", args.tokens)) if v is not None}
    sub_ok = not args.no_subs and not args.skip_e2e and not over and args.emulate_tp == 1
    clocks = ClockSampler(local).__enter__()

    head = Offload(rk, args.workload, over)
    config = head.config()
    device = head.device_step(args.steps, args.warmup)
    block_hash = head.hash_kernel(args.steps, args.warmup)
    link = e2e = None
    disk = server = layerwise = paged_layouts = noalloc = prefix = mla = tp70 = None
    host_mem = None
    if not args.skip_e2e:
        # rank 0's host copy rate around the e2e steps (the other ranks wait
        # at the link probe's first barrier): a drop says other jobs took
        # the shared host's memory bandwidth during the run
        hthreads = min(32, os.cpu_count() or 1)
        if rank == 0:
            host_mem = {"threads": hthreads, "copy_gbs_before_e2e": host_copy_gbs(hthreads)}
        link = link_probe(rk, args.link_seconds)
        threads = tuple(int(x) for x in args.duplex_threads.split(",")) if args.duplex_threads else None
        e2e = head.e2e(args.steps, args.warmup, budget, threads)
        if rank == 0:
            host_mem["copy_gbs_after_e2e"] = host_copy_gbs(hthreads)
    s = dict(dev=dev, nrec=head.nrec, rec_bytes=head.rec_bytes, bpc=head.bpc, n_blocks=head.n_blocks,
             unit=head.unit, disjoint=head.disjoint, local=local, world=world, rank=rank, n_req=head.n_req,
             n_tok=head.n_tok, per_req_blocks=head.prb, payload=head.payload)
    # on the headline shapes only: both hold every record in HBM beside the
    # paged cache (two copies for the paged-layout probe), which the 80-layer
    # preset's records (80 GiB at N = 1) do not leave room for
    if world == 1 and args.emulate_tp == 1 and args.workload == "llama3-8b":
        b_save = torch.from_numpy(head.bt_save.astype(np.int64)).to(dev)
        b_load = torch.from_numpy(head.bt_load.astype(np.int64)).to(dev)
        paged_layouts = _paged_layout_probe(args, head.layers, b_save, b_load, s)
        del b_save, b_load
        if not over:
            noalloc = head.noalloc_step(args.steps, args.warmup)
    if not args.skip_e2e and (args.disk_dir or args.layerwise or args.via_server):
        hashes = np.zeros((head.nblk, 32), dtype=np.uint8)
        n = lib.kv_block_hash_host(local, np.ascontiguousarray(head.tokens.reshape(-1)).ctypes.data,
                                   np.full(head.n_req, head.n_tok, dtype=np.int64).ctypes.data, head.n_req, BS,
                                   _sha_none(), hashes.ctypes.data)
        assert n == head.nblk
        if args.disk_dir:
            disk = _disk_tier_probe(args, cc, lib, head.layers, head.layout, head.kp, head.vp, hashes, head.bt_save,
                                    head.bt_load, head.disjoint, s)
        if args.layerwise and world == 1:
            layerwise = _layerwise_probe(args, cc, head.layers, head.layout, head.kp, head.vp, hashes,
                                         head.bt_save, head.bt_load, s)
        if args.via_server and world == 1:
            server = _server_probe(args, head.layers, hashes, head.bt_save, head.bt_load, head.disjoint, s)
    if sub_ok and world == 1 and args.workload == "llama3-8b":
        prefix = _sub_line(_prefix_reuse(dev, cc, lib, args.sub_steps, args.sub_warmup, layers=head.layers),
                           ("value", "unit", "workload", "steps", "warmup", "ms_per_step", "hit_blocks_per_request",
                            "hit_rate_chunks", "records_stored_per_step", "store_keys_deduplicated_per_step",
                            "save_gbs", "load_gbs", "p50_load_latency_ms", "verified_bytes"))
    head.free()
    del head
    if sub_ok and world == 1:
        from oracle.cache_model import LRUPool     # host-side LRU model: the checker only
        mla = _sub_line(_mla_evict(dev, cc, lib, LRUPool, args.sub_steps, args.sub_warmup),
                        ("value", "unit", "workload", "steps", "warmup", "ms_per_step", "pool_records",
                         "working_set_records", "hit_rate_chunks", "evictions_per_pass", "hits_per_pass",
                         "lru_model_hits", "lru_model_evictions", "hits_match_model", "evictions_match_model",
                         "save_gbs", "load_gbs", "p50_load_latency_ms", "loaded_block_mismatches",
                         "verified_bytes"))
    if sub_ok and args.workload == "llama3-8b":
        big = Offload(rk, "tp70b")
        tp70 = {"config": big.config(), "device": big.device_step(args.sub_steps, args.sub_warmup),
                "e2e": big.e2e(args.sub_steps, args.sub_warmup, budget)}
        big.free()
        del big
    clocks.__exit__(None, None, None)
    cpu = None
    if host_mem is not None and sub_ok:
        host_mem["copy_gbs_after_other_configs"] = host_copy_gbs(host_mem["threads"])
    if rank == 0 and world == 1 and args.cpu_seconds > 0 and args.emulate_tp == 1:
        cpu = cpu_sample_run("port", args.cpu_seconds, None, os.cpu_count() or 1)
        cpu.pop("times_s", None)
        # the reference's own concurrency: 4 CaCopy threads (src/cache/cache.c:777)
        four = cpu_sample_run("port", args.cpu_seconds / 2, None, 4)
        cpu["value_4_threads"] = round(four["value"], 3)
        cpu["cpu_model"] = _cpu_model()
        # each other configuration's CPU path at its own geometry, ~2 GiB per direction
        nth, sub_s = os.cpu_count() or 1, args.cpu_seconds / 4
        if prefix:
            prefix["cpu_baseline"] = cpu_geometry_sample("prefix reuse (Llama-3-8B geometry)", L,
                                                         KV_HEADS * HEAD_DIM * ELT, BS, 2, 64, nth, sub_s)
        if tp70:
            tp70["cpu_baseline"] = cpu_geometry_sample("Llama-3-70B, TP = 1", PRESETS["tp70b"]["layers"],
                                                       KV_HEADS * HEAD_DIM * ELT, BS, 2, 24, nth, sub_s)
        if mla:
            mla["cpu_baseline"] = cpu_geometry_sample("DeepSeek-V2-Lite MLA latent", 27, 576 * 2, 64, 1, 256,
                                                      nth, sub_s)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    dup = e2e.get("duplex") if e2e else None
    seq = e2e.get("sequential") if e2e else None
    if seq and "skipped" in seq:
        seq = None
    head_e2e = dup or seq
    if link and head_e2e:
        if seq:
            seq["save_frac_of_link"] = round(seq["save_gbs_aggregate"] / link["d2h"]["aggregate"], 4)
            seq["load_frac_of_link"] = round(seq["load_gbs_aggregate"] / link["h2d"]["aggregate"], 4)
        if dup:
            dup["frac_of_link_both_directions"] = round(dup["value"] / link["both"]["aggregate"], 4)
    if tp70 and link:
        t_seq, t_dup = tp70["e2e"].get("sequential"), tp70["e2e"].get("duplex")
        if t_seq and "skipped" not in t_seq:
            t_seq["save_frac_of_link"] = round(t_seq["save_gbs_aggregate"] / link["d2h"]["aggregate"], 4)
            t_seq["load_frac_of_link"] = round(t_seq["load_gbs_aggregate"] / link["h2d"]["aggregate"], 4)
        if t_dup:
            t_dup["frac_of_link_both_directions"] = round(t_dup["value"] / link["both"]["aggregate"], 4)
    if head_e2e:
        value, ms = head_e2e["value"], head_e2e["ms_per_step"]
        launches = head_e2e["gpu_launches"]
        # the metric's latency: one request's load with the link to itself
        # (sequential step); the duplex step's, with other transfers in
        # flight, is reported beside it
        p50 = (seq or head_e2e)["p50_load_latency_ms"]
        e2e_line = {"value": value, "unit": "GB/s", "mode": "duplex" if dup else "sequential",
                    "h2d_bytes_per_step": head_e2e["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": head_e2e["d2h_bytes_per_step"],
                    "bytes_note": "per rank per step: KV payload + token ids + block tables up, payload + block "
                                  "hashes down",
                    "ms_per_step": ms, "p50_load_latency_ms": p50,
                    "p50_load_latency_under_duplex_ms": dup["p50_load_latency_ms"] if dup else None,
                    "latency_note": "p50_load_latency_ms: one request's load (cache_load of its records) with "
                                    "the host link to itself (sequential step); under_duplex: the value "
                                    "step's loads, with another load and a save in flight",
                    "requests_per_step": head_e2e["requests_per_step"], "verified_bytes": head_e2e["verified_bytes"]}
    else:
        value, ms, launches, p50 = device["value"], device["ms_per_step"], device["launches"], None
        e2e_line = e2e
    verified = [device["verified_bytes"]] + [x["verified_bytes"] for x in (seq, dup) if x]
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded N(0,1) bf16 KV, uniform token ids, random block tables)",
        "config": config,
        "value_kind": ("save+load payload through cache_store / cache_load, KV in HBM <-> pinned host pool, "
                       f"{'duplex' if dup else 'sequential'} step" if head_e2e else "device kernels only"),
        "e2e": e2e_line, "sequential": seq, "duplex": dup, "link": link,
        "p50_load_latency_ms": p50, "device": device, "roofline": device["roofline"],
        "block_hash": block_hash, "tp70b": tp70, "prefix_reuse": prefix, "mla_evict": mla,
        "noalloc": noalloc, "paged_layouts": paged_layouts,
        "disk_tier": disk, "via_server": server, "layerwise": layerwise,
        "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": clocks.summary(), "host": hinfo,
        "host_memory": host_mem,
        "pool_budget_gib_per_rank": round(budget / 2**30, 1),
        "verified_bytes": all(verified),
    }
    if args.emulate_tp != 1:
        config["workload"] += f" (1 process emulating rank 0 of TP={args.emulate_tp})"
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
