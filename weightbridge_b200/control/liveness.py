"""Peer liveness: notice at once that a process of the session is gone.

Every sender keeps one TCP connection to each receiver worker it sends to.  A process that
exits - cleanly or not - has its sockets closed by the OS, so the other end reads EOF; an
orderly disconnect first sends ``bye``.  EOF without ``bye`` means the peer died, and the
watcher reports it: a receiver then publishes the error in the ``done`` keys it waits on,
a sender in the ``ready`` / ``pulled`` keys it waits on, so the blocked wait returns with a
``PeerError`` within milliseconds instead of running into the sync deadline.  A peer that is
alive but stuck is still caught by the deadline.  The reference has no failure detection
beyond HTTP status codes (``wbridge/backend/direct_sender.py:87, 113, 190``).
"""
from __future__ import annotations

import logging
import select
import socket
import struct
import threading
from typing import Callable

logger = logging.getLogger(__name__)

BYE = b"bye"


class PeerWatch:
    """A thread watching the connections to the session's peers (and, on the receiver side,
    accepting them on ``listener``).  ``on_lost(peer)`` runs on that thread."""

    def __init__(self, on_lost: Callable[[int], None], listener: socket.socket | None = None):
        self._on_lost = on_lost
        self._listener = listener
        self._conns: dict[socket.socket, int] = {}
        self._bye: set[int] = set()
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self.lost: list[int] = []
        self._thread = threading.Thread(target=self._run, name="wbridge-liveness", daemon=True)
        self._thread.start()

    @staticmethod
    def listen(host: str) -> tuple[socket.socket, int]:
        s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        s.bind((host, 0))
        s.listen(64)
        return s, s.getsockname()[1]

    @staticmethod
    def connect(host: str, port: int, me: int, timeout_s: float) -> socket.socket:
        s = socket.create_connection((host, port), timeout=timeout_s)
        s.sendall(struct.pack("<q", me))
        s.settimeout(None)
        return s

    def add(self, sock: socket.socket, peer: int) -> None:
        with self._lock:
            self._conns[sock] = peer

    def _accept(self) -> None:
        conn, _addr = self._listener.accept()
        conn.settimeout(5.0)
        try:
            buf = b""
            while len(buf) < 8:
                chunk = conn.recv(8 - len(buf))
                if not chunk:
                    raise ConnectionError("closed before naming itself")
                buf += chunk
        except (OSError, ConnectionError):
            conn.close()
            return
        conn.settimeout(None)
        self.add(conn, struct.unpack("<q", buf)[0])

    def _run(self) -> None:
        while not self._stop.is_set():
            with self._lock:
                socks = list(self._conns)
            watch = socks + ([self._listener] if self._listener is not None else [])
            if not watch:
                self._stop.wait(0.2)
                continue
            try:
                ready, _, _ = select.select(watch, [], [], 0.2)
            except (OSError, ValueError):      # a socket closed under us (teardown)
                continue
            for s in ready:
                if s is self._listener:
                    try:
                        self._accept()
                    except OSError:
                        pass
                    continue
                try:
                    data = s.recv(64)
                except OSError:
                    data = b""
                with self._lock:
                    peer = self._conns.get(s)
                if peer is None:
                    continue
                if data and BYE in data:
                    self._bye.add(peer)
                if data:
                    continue
                with self._lock:
                    self._conns.pop(s, None)
                s.close()
                if peer in self._bye or self._stop.is_set():
                    continue
                self.lost.append(peer)
                try:
                    self._on_lost(peer)
                except Exception:
                    logger.exception("liveness callback for peer %d", peer)

    def close(self) -> None:
        """Say ``bye`` on every connection and stop watching."""
        self._stop.set()
        with self._lock:
            socks = list(self._conns)
            self._conns.clear()
        for s in socks:
            try:
                s.sendall(BYE)
            except OSError:
                pass
            try:
                s.close()
            except OSError:
                pass
        if self._listener is not None:
            try:
                self._listener.close()
            except OSError:
                pass
        self._thread.join(2.0)
