"""Passing file descriptors between processes of one node (SCM_RIGHTS over a Unix socket).

VMM allocations and NVLink multicast objects are shared as POSIX file descriptors
(``cuMemExportToShareableHandle``); a descriptor only means something inside the process
that owns it, so it travels over a Unix-domain socket as ancillary data.  ``FdServer``
serves named descriptors from one process; ``fetch_fd`` gets one from another process.
The socket lives in the abstract namespace (no file to clean up).
"""
from __future__ import annotations

import os
import socket
import threading
import uuid


class FdServer:
    def __init__(self):
        self.address = f"\0wbridge-fd-{os.getpid()}-{uuid.uuid4().hex[:12]}"
        self._fds: dict[str, int] = {}
        self._lock = threading.Lock()
        self._sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self._sock.bind(self.address)
        self._sock.listen(64)
        self._sock.settimeout(0.2)
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._serve, name="wbridge-fd-server", daemon=True)
        self._thread.start()

    def publish(self, key: str, fd: int) -> None:
        with self._lock:
            self._fds[key] = fd

    def _serve(self) -> None:
        while not self._stop.is_set():
            try:
                conn, _ = self._sock.accept()
            except (socket.timeout, OSError):
                continue
            with conn:
                conn.settimeout(5.0)
                try:
                    key = conn.recv(256).decode()
                    with self._lock:
                        fd = self._fds.get(key)
                    if fd is None:
                        conn.sendall(b"\x00")
                    else:
                        socket.send_fds(conn, [b"\x01"], [fd])
                except OSError:
                    pass

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2)
        self._sock.close()


def fetch_fd(address: str, key: str, timeout_s: float = 10.0) -> int:
    """A duplicate (in this process) of the descriptor ``key`` served at ``address``."""
    with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
        s.settimeout(timeout_s)
        s.connect(address)
        s.sendall(key.encode())
        msg, fds, _flags, _addr = socket.recv_fds(s, 16, 1)
        if msg[:1] != b"\x01" or not fds:
            raise KeyError(f"no descriptor {key!r} served at {address!r}")
        return fds[0]
