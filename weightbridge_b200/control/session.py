"""Session store: a TCPStore that sender rank 0 hosts for one connect.

Holds the rendezvous of the senders and receivers of a session (the reference builds a
joint NCCL/gloo process group for this, ``wbridge/utils/distributed.py:28-82``): receiver
bindings and IPC handles, the source assignment, plan digests, and the per-sync
``ready`` / ``done`` handshakes.  Every wait is bounded.
"""
from __future__ import annotations

import json
import os
import socket
import zlib
from datetime import timedelta
from typing import Any, Iterable

import torch.distributed as dist


class SessionTimeout(TimeoutError):
    pass


class PeerError(RuntimeError):
    """A peer of the session published an error instead of the key we wait for."""


# A failing peer stores this prefix + its message in the keys others wait on, so a single
# blocking wait returns and the waiter raises instead of sitting out its deadline.
ERROR_PREFIX = b"!error:"


class Session:
    def __init__(self, host: str, port: int, is_master: bool, timeout_s: float, prefix: str = "wbridge"):
        self.timeout_s = timeout_s
        self._tcp = dist.TCPStore(host, port, is_master=is_master, timeout=timedelta(seconds=timeout_s),
                                  wait_for_workers=False)
        self.port = self._tcp.port
        self.host = host
        self.prefix = prefix
        self.store = dist.PrefixStore(prefix, self._tcp)
        self._cur_timeout = timeout_s

    def set(self, key: str, value: bytes | str) -> None:
        self.store.set(key, value)

    CHUNK = 4 << 20          # TCPStore caps one value at 8 MiB

    def set_json(self, key: str, obj: Any) -> None:
        """Store ``obj`` as zlib-compressed JSON, split in chunks when it is large (a receiver
        binding of a 19k-tensor MoE model is ~12 MB of JSON)."""
        blob = zlib.compress(json.dumps(obj, separators=(",", ":")).encode(), 1)
        n = (len(blob) + self.CHUNK - 1) // self.CHUNK
        for i in range(n):
            self.store.set(f"{key}#{i}", blob[i * self.CHUNK:(i + 1) * self.CHUNK])
        self.store.set(key, f"z:{n}")

    def wait(self, keys: Iterable[str], timeout_s: float | None = None, what: str = "") -> None:
        keys = list(keys)
        if not keys:
            return
        t = timeout_s if timeout_s is not None else self.timeout_s
        try:
            self.store.wait(keys, timedelta(seconds=t))
        except Exception as e:  # torch raises DistStoreError / RuntimeError on timeout
            raise SessionTimeout(f"timed out after {t:.1f}s waiting for {what or keys[:4]}: {e}") from None

    def get(self, key: str, timeout_s: float | None = None) -> bytes:
        self.wait([key], timeout_s, key)
        return self.store.get(key)

    def get_json(self, key: str, timeout_s: float | None = None) -> Any:
        head = self.get(key, timeout_s)
        if head.startswith(ERROR_PREFIX):
            raise PeerError(head[len(ERROR_PREFIX):].decode(errors="replace"))
        head = head.decode()
        if not head.startswith("z:"):
            return json.loads(head)
        n = int(head[2:])
        blob = b"".join(self.store.get(f"{key}#{i}") for i in range(n))
        return json.loads(zlib.decompress(blob))

    def wait_checked(self, keys: Iterable[str], timeout_s: float | None = None, what: str = "") -> list[bytes]:
        """Wait for ``keys`` (one blocking call) and raise ``PeerError`` if a peer stored an
        error in any of them instead of a value."""
        keys = list(keys)
        if not keys:
            return []
        t = timeout_s if timeout_s is not None else self.timeout_s
        if t != self._cur_timeout:          # multi_get blocks until every key exists, up to this
            self.store.set_timeout(timedelta(seconds=t))
            self._cur_timeout = t
        try:
            vals = self.store.multi_get(keys)   # one round trip: wait and read
        except Exception as e:
            raise SessionTimeout(f"timed out after {t:.1f}s waiting for {what or keys[:4]}: {e}") from None
        for k, v in zip(keys, vals):
            if v.startswith(ERROR_PREFIX):
                raise PeerError(v[len(ERROR_PREFIX):].decode(errors="replace"))
        return vals

    def raise_posted_error(self, keys: Iterable[str]) -> None:
        """Raise ``PeerError`` if a peer posted an error in any of ``keys`` (non-blocking; a
        key that does not exist yet is no error)."""
        for k in keys:
            if self.store.check([k]):
                v = self.store.get(k)
                if v.startswith(ERROR_PREFIX):
                    raise PeerError(v[len(ERROR_PREFIX):].decode(errors="replace"))

    def set_error(self, keys: Iterable[str], message: str) -> None:
        """Publish a failure in the keys a peer is (or will be) waiting for."""
        for k in keys:
            try:
                self.store.set(k, ERROR_PREFIX + message.encode())
            except Exception:
                pass

    def multi_set(self, keys: list[str], values: list[bytes | str]) -> None:
        if keys:
            self.store.multi_set(keys, [v if isinstance(v, bytes) else v.encode() for v in values])

    def check(self, key: str) -> bool:
        return self.store.check([key])

    def add(self, key: str, n: int) -> int:
        return self.store.add(key, n)

    def delete(self, key: str) -> None:
        try:
            self.store.delete_key(key)
        except Exception:
            pass


class Janitor:
    """A thread with a store client of its own for work that must not wait behind (or block)
    the main client: deleting finished handshake keys (one round trip each, kept off the next
    sync's critical path) and publishing errors while the main thread may be blocked in a
    wait on the same session."""

    def __init__(self, host: str, port: int, timeout_s: float, prefix: str = "wbridge"):
        import queue
        import threading
        self._args = (host, port, timeout_s, prefix)
        self._q: "queue.SimpleQueue[tuple | None]" = queue.SimpleQueue()
        self._thread = threading.Thread(target=self._run, name="wbridge-janitor", daemon=True)
        self._thread.start()

    def delete(self, keys: list[str]) -> None:
        if keys:
            self._q.put(("delete", list(keys), None))

    def set_error(self, keys: list[str], message: str) -> None:
        if keys:
            self._q.put(("error", list(keys), message))

    def _run(self) -> None:
        sess = None
        while True:
            job = self._q.get()
            if job is None:
                return
            kind, keys, message = job
            try:
                if sess is None:
                    host, port, timeout_s, prefix = self._args
                    sess = Session(host, port, is_master=False, timeout_s=timeout_s, prefix=prefix)
                if kind == "delete":
                    for k in keys:
                        sess.delete(k)
                else:
                    sess.set_error(keys, message)
            except Exception:
                pass             # the session is gone: nothing left to clean or tell

    def close(self, timeout_s: float = 2.0) -> None:
        self._q.put(None)
        self._thread.join(timeout_s)


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def host_address() -> str:
    """The address other hosts reach this one at: ``WBRIDGE_HOST_ADDRESS`` if set, else the
    address of the default route, else loopback."""
    env = os.environ.get("WBRIDGE_HOST_ADDRESS")
    if env:
        return env
    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
            s.connect(("10.255.255.255", 1))
            return s.getsockname()[0]
    except OSError:
        return "127.0.0.1"


def local_address() -> str:
    """The session store's address on sender rank 0: ``WBRIDGE_MASTER_ADDRESS`` if set, else
    this host's address (``host_address``)."""
    env = os.environ.get("WBRIDGE_MASTER_ADDRESS")
    return env if env else host_address()
