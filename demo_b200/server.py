"""CrossCache server: the ZeroMQ front-end of the cache manager, serving the
reference's wire protocol (src/main.c; messages in demo_b200/protocol.py).

    python -m demo_b200.server [-P 5555] [--chunksize 256] [--cachedir DIR]
                               [--poolsize BYTES] [--backend cuda|mem]

Same behaviour as main.c:
  - a ROUTER socket on tcp://*:<port>; every request frame is answered with
    one msg_response (uid, ok) to the sender's identity      (main.c:490-547)
  - worker slots indexed by the message's node_id (0-7); a REGISTER on a
    taken slot unregisters the old worker first         (main.c:58-121, 244-290)
  - LOOKUP asks rank 0 of (model, world_size) and answers hit keys *
    chunk_size tokens                                          (main.c:126-141)
  - STORE / LOAD on the registered slot; unknown slot -EINVAL   (main.c:143-190)
  - register/unregister/lookup run on a 2-thread pool, stores and loads on
    4-thread pools each                                        (main.c:388-413)
Differences: the socket is owned by one thread and handlers hand their
replies back to it (the reference sends from every pool thread under a
spinlock); a message whose lengths do not add up, or a STORE/LOAD whose key
count does not match its block count, is answered -EINVAL (the reference
reads past the frame or aborts on sys_assert); node_id is also the CUDA
device whose memory the worker's IPC keys name, so the server must see the
same device numbering as its workers.
"""
from __future__ import annotations

import argparse
import ctypes as C
import errno
import json
import logging
import os
import queue
import signal
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import cache as cc
from . import protocol as P
from ._lib import CACHE_BACKEND_CUDA, CACHE_BACKEND_MEM, ModelInfo, WorkerContext, lib

MAX_NODE_NUM = 8
logger = logging.getLogger(__name__)


class CacheServer:
    def __init__(self, bind: str = "tcp://*:5555", chunk_size: int = 256, pool_size: int = 4 << 30,
                 cache_dir: str | None = None, backend: int = CACHE_BACKEND_CUDA,
                 common_threads: int = 2, store_threads: int = 4, load_threads: int = 4, context=None):
        import zmq

        self._zmq = zmq
        self.bind = bind
        self.chunk_size = chunk_size
        self.pool_size = pool_size
        self.cache_dir = cache_dir
        self.backend = backend
        self._ctx = context or zmq.Context.instance()
        self._threads = (common_threads, store_threads, load_threads)
        self._slots: list[cc.Worker | None] = [None] * MAX_NODE_NUM
        self._slot_lock = threading.Lock()
        self._replies: queue.SimpleQueue = queue.SimpleQueue()
        self._wake_r, self._wake_w = os.pipe()
        self._stop = threading.Event()
        self._closing = False
        self._loop_thread: threading.Thread | None = None
        self._sock = None
        self.endpoint: str | None = None
        self.requests = 0

    # ---- lifecycle -----------------------------------------------------
    def start(self) -> "CacheServer":
        cc.init(self.chunk_size, self.pool_size, self.cache_dir or None, self.backend)
        try:
            self._sock = self._ctx.socket(self._zmq.ROUTER)
            self._sock.setsockopt(self._zmq.LINGER, 0)
            self._sock.bind(self.bind)
            self.endpoint = self._sock.getsockopt_string(self._zmq.LAST_ENDPOINT)
        except Exception:
            if self._sock is not None:
                self._sock.close()
            cc.exit()
            raise
        c, s, ld = self._threads
        self._common = ThreadPoolExecutor(c, thread_name_prefix="CommThp")
        self._store = ThreadPoolExecutor(s, thread_name_prefix="StoreThp")
        self._load = ThreadPoolExecutor(ld, thread_name_prefix="LoadThp")
        self._loop_thread = threading.Thread(target=self._loop, name="CrossCacheServer", daemon=True)
        self._loop_thread.start()
        logger.info("CrossCache listening on %s, chunk_size:%u, cachedir:%s", self.endpoint,
                    self.chunk_size, self.cache_dir)
        return self

    def stop(self) -> None:
        if self._loop_thread is None:
            return
        # new requests are refused; the ones in the pools finish and are
        # answered by the loop before it leaves
        self._closing = True
        for pool in (self._common, self._store, self._load):
            pool.shutdown(wait=True)
        self._stop.set()
        os.write(self._wake_w, b"x")
        self._loop_thread.join()
        self._loop_thread = None
        with self._slot_lock:
            for i, w in enumerate(self._slots):
                if w is not None:
                    _log_worker_stats(i, w, "server stopped")
                    w.unregister()
                    self._slots[i] = None
        self._sock.close()
        cc.exit()
        os.close(self._wake_r)
        os.close(self._wake_w)

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()

    # ---- socket loop ---------------------------------------------------
    def _loop(self) -> None:
        zmq = self._zmq
        poller = zmq.Poller()
        poller.register(self._sock, zmq.POLLIN)
        poller.register(self._wake_r, zmq.POLLIN)
        while True:
            events = dict(poller.poll(1000))
            if self._wake_r in events:
                os.read(self._wake_r, 4096)
            self._flush_replies()
            if self._stop.is_set():
                return
            if events.get(self._sock) == zmq.POLLIN:
                while True:
                    try:
                        frames = self._sock.recv_multipart(zmq.NOBLOCK)
                    except zmq.Again:
                        break
                    self._dispatch(frames)

    def _flush_replies(self) -> None:
        while True:
            try:
                ident, frame = self._replies.get_nowait()
            except queue.Empty:
                return
            self._sock.send_multipart([ident, frame])

    def _reply(self, ident: bytes, uid: int, ret: int) -> None:
        self._replies.put((ident, P.encode_response(uid, ret)))
        os.write(self._wake_w, b"x")

    def _dispatch(self, frames: list[bytes]) -> None:
        self.requests += 1
        if len(frames) != 2:
            logger.error("dropping a message of %d frames", len(frames))
            return
        ident, body = frames
        try:
            msg = P.decode_request(body)
        except P.ProtocolError as e:
            logger.error("bad request: %s", e)
            if hasattr(e, "uid"):
                self._reply(ident, e.uid, -errno.EINVAL)
            return
        if isinstance(msg, (P.Register, P.Unregister, P.Lookup)):
            pool = self._common
        else:
            pool = self._store if msg.op == P.Op.STORE else self._load
        if self._closing:
            self._reply(ident, msg.uid, -errno.ESHUTDOWN)
            return
        try:
            pool.submit(self._handle, ident, msg)
        except RuntimeError:              # pool already shut down
            self._reply(ident, msg.uid, -errno.ESHUTDOWN)

    def _handle(self, ident: bytes, msg) -> None:
        t0 = time.perf_counter()
        try:
            if isinstance(msg, P.Register):
                ret = self._register(msg)
            elif isinstance(msg, P.Unregister):
                ret = self._unregister(msg.node_id)
            elif isinstance(msg, P.Lookup):
                ret = self._lookup(msg)
            else:
                ret = self._transfer(msg)
        except Exception:                 # answered, never left hanging
            logger.exception("request uid %d failed", msg.uid)
            ret = -errno.EIO
        if logger.isEnabledFor(logging.DEBUG):
            logger.debug("%s worker:%u uid:%u keys:%d -> %d (%.2f ms)", type(msg).__name__ if not isinstance(
                msg, P.Transfer) else msg.op.name, msg.node_id, msg.uid, getattr(msg, "keys_num", 0), ret,
                (time.perf_counter() - t0) * 1e3)
        self._reply(ident, msg.uid, ret)

    # ---- operations (main.c:58-190) ------------------------------------
    def _register(self, m: P.Register) -> int:
        if m.node_id >= MAX_NODE_NUM:
            return -errno.ERANGE
        layout = cc.KVLayout(m.num_layers, m.num_blocks, m.block_size, m.hidden_dim_size, m.element_size,
                             2 if m.v_keys is not None else 1, m.block_stride, m.head_bytes)
        w = cc.Worker.from_keys(m.model_name, layout, m.k_keys, m.v_keys, m.key_len, node_id=m.node_id,
                                world_size=m.world_size, rank=m.rank_id)
        with self._slot_lock:
            old = self._slots[m.node_id]
            if old is not None:
                logger.warning("worker:%u updated", m.node_id)
                old.unregister()
                self._slots[m.node_id] = None
            try:
                w.register()
            except cc.CacheError as e:
                return e.ret
            self._slots[m.node_id] = w
        return 0

    def _unregister(self, nid: int) -> int:
        if nid >= MAX_NODE_NUM:
            return -errno.ERANGE
        with self._slot_lock:
            w = self._slots[nid]
            self._slots[nid] = None
        if w is None:
            logger.warning("worker:%u has not registered", nid)
            return 0
        _log_worker_stats(nid, w, "unregistered")
        w.unregister()
        return 0

    def _lookup(self, m: P.Lookup) -> int:
        if not m.keys_num or m.key_len < cc.KEY_LEN:
            return 0
        ctx = WorkerContext()
        name = m.model_name.encode()
        ctx.model = ModelInfo(name, 0, 0, 0)
        ctx.world_size = m.world_size
        ctx.rank_id = 0                     # main.c:136: rank 0 answers for the group
        hit = lib.cache_lookup(C.byref(ctx), m.keys, m.keys_num, m.key_len)
        return (hit // m.key_len) * self.chunk_size

    def _transfer(self, m: P.Transfer) -> int:
        if m.node_id >= MAX_NODE_NUM:
            return -errno.ERANGE
        with self._slot_lock:
            w = self._slots[m.node_id]
        if w is None:
            logger.warning("worker:%u has not been registered", m.node_id)
            return -errno.EINVAL
        bs = w.layout.block_size
        if m.keys_num * self.chunk_size != len(m.block_ids) * bs or m.key_len < cc.KEY_LEN:
            return -errno.EINVAL
        bids = np.ascontiguousarray(m.block_ids, dtype=np.uint64)
        fn = lib.cache_store if m.op == P.Op.STORE else lib.cache_load
        return fn(C.byref(w.ctx), m.keys, m.key_len, bids.ctypes.data, len(bids))


def _log_worker_stats(nid: int, w: cc.Worker, why: str) -> None:
    """one INFO line per departing worker: its entry's counters as JSON"""
    try:
        st = w.stats()
    except cc.CacheError:
        return
    ctx = w.ctx
    logger.info("worker:%u %s: model=%s tp=%u rank=%u stats=%s", nid, why, ctx.model.model_name.decode(),
                ctx.world_size, ctx.rank_id, json.dumps(st, sort_keys=True))


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description="CrossCache server (src/main.c options)")
    ap.add_argument("-P", "--port", type=int, default=5555)
    ap.add_argument("--chunksize", type=int, default=256)
    ap.add_argument("--cachedir", default="/var/log/crosscache",
                    help="disk-tier directory (main.c default); '' for memory only")
    ap.add_argument("--poolsize", type=int, default=4 << 30, help="pinned bytes per registered worker")
    ap.add_argument("--backend", choices=["cuda", "mem"], default="cuda")
    ap.add_argument("--host", default="*", help="interface to bind")
    args = ap.parse_args(argv)
    logging.basicConfig(level=os.environ.get("CROSSCACHE_PYLOG", "INFO"))
    srv = CacheServer(f"tcp://{args.host}:{args.port}", args.chunksize, args.poolsize, args.cachedir or None,
                      CACHE_BACKEND_CUDA if args.backend == "cuda" else CACHE_BACKEND_MEM)
    srv.start()
    done = threading.Event()
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, lambda *_: done.set())
    done.wait()
    srv.stop()


if __name__ == "__main__":
    main()
