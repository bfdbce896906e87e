"""Client side of the CrossCache server connection (python/utils/mq.py:14-117):
a DEALER socket, requests answered through futures keyed by a per-client
request uid.

The reference sends from one thread and receives from another on the same
socket; ZeroMQ sockets are not thread-safe, so here one IO thread owns the
socket and callers hand it frames through a queue (woken by a pipe).
"""
from __future__ import annotations

import itertools
import os
import queue
import threading
from concurrent.futures import Future
from typing import Callable

from . import protocol as P


class MessageQueueClient:
    def __init__(self, server_url: str, context=None):
        import zmq

        self._zmq = zmq
        self._ctx = context or zmq.Context.instance()
        self._sock = self._ctx.socket(zmq.DEALER)
        self._sock.setsockopt(zmq.LINGER, 0)
        self._sock.connect(server_url)
        self._out: queue.SimpleQueue = queue.SimpleQueue()
        self._pending: dict[int, Future] = {}
        self._lock = threading.Lock()
        self._uids = itertools.count()
        self._wake_r, self._wake_w = os.pipe()
        self._stop = threading.Event()
        self._io = threading.Thread(target=self._loop, name="CrossCacheClient", daemon=True)
        self._io.start()

    def submit(self, build: Callable[[int], bytes]) -> Future:
        """build(uid) -> request frame; the future receives the signed
        status of the response."""
        fut: Future = Future()
        with self._lock:
            if self._stop.is_set():
                raise RuntimeError("client closed")
            uid = next(self._uids) & 0xFFFFFFFF
            self._pending[uid] = fut
        try:
            frame = build(uid)
        except Exception:
            with self._lock:
                self._pending.pop(uid, None)
            raise
        self._out.put(frame)
        os.write(self._wake_w, b"x")
        return fut

    def request(self, build: Callable[[int], bytes], timeout: float | None = None) -> int:
        return self.submit(build).result(timeout=timeout)

    def _loop(self) -> None:
        zmq = self._zmq
        poller = zmq.Poller()
        poller.register(self._sock, zmq.POLLIN)
        poller.register(self._wake_r, zmq.POLLIN)
        while not self._stop.is_set():
            events = dict(poller.poll(1000))
            if self._wake_r in events:
                os.read(self._wake_r, 4096)
            while True:
                try:
                    frame = self._out.get_nowait()
                except queue.Empty:
                    break
                self._sock.send(frame)
            if events.get(self._sock) == zmq.POLLIN:
                while True:
                    try:
                        msg = self._sock.recv(zmq.NOBLOCK)
                    except zmq.Again:
                        break
                    try:
                        uid, status = P.decode_response(msg)
                    except P.ProtocolError:
                        continue
                    with self._lock:
                        fut = self._pending.pop(uid, None)
                    if fut is not None:
                        fut.set_result(status)

    def close(self) -> None:
        with self._lock:
            self._stop.set()
            pending = list(self._pending.values())
            self._pending.clear()
        os.write(self._wake_w, b"x")
        self._io.join()
        for fut in pending:
            if not fut.done():
                fut.set_exception(ConnectionAbortedError("client closed before the server answered"))
        self._sock.close()
        os.close(self._wake_r)
        os.close(self._wake_w)
