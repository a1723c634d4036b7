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
import time
import zlib
from datetime import timedelta
from typing import Any, Iterable

import torch.distributed as dist


class SessionTimeout(TimeoutError):
    pass


class PeerError(RuntimeError):
    """A peer of the session published an error instead of the key we wait for."""


class Session:
    def __init__(self, host: str, port: int, is_master: bool, timeout_s: float, prefix: str = "wbridge"):
        self.timeout_s = timeout_s
        self._tcp = dist.TCPStore(host, port, is_master=is_master, timeout=timedelta(seconds=timeout_s),
                                  wait_for_workers=False)
        self.port = self._tcp.port
        self.host = host
        self.store = dist.PrefixStore(prefix, self._tcp)

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

    def get_json(self, key: str, timeout_s: float | None = None, error_key: str | None = None) -> Any:
        head = (self.get_or_error(key, error_key, timeout_s) if error_key else self.get(key, timeout_s)).decode()
        if not head.startswith("z:"):
            return json.loads(head)
        n = int(head[2:])
        blob = b"".join(self.store.get(f"{key}#{i}") for i in range(n))
        return json.loads(zlib.decompress(blob))

    def get_or_error(self, key: str, error_key: str, timeout_s: float | None = None) -> bytes:
        """Wait for ``key`` but fail fast when the peer publishes ``error_key`` instead."""
        t = timeout_s if timeout_s is not None else self.timeout_s
        deadline = time.monotonic() + t
        while True:
            left = deadline - time.monotonic()
            try:
                self.store.wait([key], timedelta(seconds=max(0.01, min(0.5, left))))
                return self.store.get(key)
            except Exception:
                pass
            if self.store.check([error_key]):
                raise PeerError(self.store.get(error_key).decode())
            if time.monotonic() >= deadline:
                raise SessionTimeout(f"timed out after {t:.1f}s waiting for {key}")

    def wait_or_error(self, keys: Iterable[str], error_keys: Iterable[str], timeout_s: float | None = None,
                      what: str = "") -> None:
        """``wait`` that also fails fast when any peer publishes one of ``error_keys``."""
        keys, error_keys = list(keys), list(error_keys)
        if not keys:
            return
        t = timeout_s if timeout_s is not None else self.timeout_s
        deadline = time.monotonic() + t
        while True:
            left = deadline - time.monotonic()
            try:
                self.store.wait(keys, timedelta(seconds=max(0.01, min(0.5, left))))
                return
            except Exception:
                pass
            for ek in error_keys:
                if self.store.check([ek]):
                    raise PeerError(self.store.get(ek).decode())
            if time.monotonic() >= deadline:
                raise SessionTimeout(f"timed out after {t:.1f}s waiting for {what or keys[:4]}")

    def check(self, key: str) -> bool:
        return self.store.check([key])

    def add(self, key: str, n: int) -> int:
        return self.store.add(key, n)

    def delete(self, key: str) -> None:
        try:
            self.store.delete_key(key)
        except Exception:
            pass


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def local_address() -> str:
    """This host's address for the session store: ``WBRIDGE_MASTER_ADDRESS`` if set, else
    the address of the default route, else loopback."""
    env = os.environ.get("WBRIDGE_MASTER_ADDRESS")
    if env:
        return env
    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
            s.connect(("10.255.255.255", 1))
            return s.getsockname()[0]
    except OSError:
        return "127.0.0.1"
