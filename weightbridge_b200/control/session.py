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
from datetime import timedelta
from typing import Any, Iterable

import torch.distributed as dist


class SessionTimeout(TimeoutError):
    pass


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

    def set_json(self, key: str, obj: Any) -> None:
        self.store.set(key, json.dumps(obj, separators=(",", ":")))

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
        return json.loads(self.get(key, timeout_s))

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
