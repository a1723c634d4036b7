"""Rollout-side HTTP control plane: FastAPI routes that fan out to the receiver workers.

Routes (on the user's FastAPI app): ``GET /wbridge/metadata``, ``POST /wbridge/connect``,
``POST /wbridge/receive``, ``GET /wbridge/stats`` (JSON) and ``GET /wbridge/metrics``
(Prometheus text format).  The controller talks to the
``WeightReceiver`` workers over a ZMQ ROUTER bound at an ``ipc://`` path; each request
carries an id and replies are matched by (worker, id), with a deadline on every gather.

Parity: ``wbridge/frontend/receiver.py:233-332`` (routes, ``set_worker_num``, per-worker
rank assignment ``base_rank + idx``, ack-before-join).  Differences: the handlers are
plain ``def`` (FastAPI runs them in its thread pool, so a slow gather never blocks the
event loop), ``worker_num`` can be given at construction, there is a synchronous
``_query_receivers_metadata`` (the reference's test calls it), and a stats route.
"""
from __future__ import annotations

import itertools
import json
import logging
import os
import tempfile
import threading
import time
from typing import Any

import zmq

from .protocol import (CONNECT_REQUEST, METADATA_REQUEST, RECEIVE_REQUEST, STATS_REQUEST, ConnectRequest)

logger = logging.getLogger(__name__)


class ControllerError(RuntimeError):
    pass


class WeightReceiverController:
    """The rollout server's side of the control plane.  ``prefix`` mounts the routes under
    ``<prefix>/wbridge/...`` so several controllers (several models) can share one app; the
    senders then use ``http://host:port<prefix>`` as the receiver URL."""

    def __init__(self, app=None, worker_num: int | None = None, timeout_s: float = 60.0, prefix: str = ""):
        fd, path = tempfile.mkstemp(prefix="wbridge_ctl_")
        os.close(fd)
        os.unlink(path)
        self._ipc_path = path
        self._ipc_name = f"ipc://{path}"
        self.timeout_s = timeout_s
        self._ctx = zmq.Context()
        self._sock = self._ctx.socket(zmq.ROUTER)
        self._sock.setsockopt(zmq.ROUTER_MANDATORY, 1)
        self._sock.setsockopt(zmq.ROUTER_HANDOVER, 1)     # a restarted worker takes over its identity
        self._sock.setsockopt(zmq.LINGER, 0)
        self._sock.bind(self._ipc_name)
        self._lock = threading.Lock()
        self._ids = itertools.count(1)
        self._worker_num: int | None = None
        self._receiver_identities: list[bytes] = []
        self.prefix = prefix.rstrip("/")
        if self.prefix and not self.prefix.startswith("/"):
            raise ValueError("prefix must start with '/'")
        if worker_num is not None:
            self.set_worker_num(worker_num)
        if app is not None:
            self.attach(app)

    def attach(self, app) -> None:
        from fastapi import APIRouter
        router = APIRouter()
        base = f"{self.prefix}/wbridge"
        router.add_api_route(f"{base}/metadata", self.get_metadata, methods=["GET"])
        router.add_api_route(f"{base}/connect", self.connect, methods=["POST"])
        router.add_api_route(f"{base}/receive", self.receive_weights, methods=["POST"])
        router.add_api_route(f"{base}/stats", self.get_stats, methods=["GET"])
        router.add_api_route(f"{base}/metrics", self.get_metrics, methods=["GET"])
        app.include_router(router)
        self.router = router

    @property
    def ipc_name(self) -> str:
        return self._ipc_name

    def set_worker_num(self, worker_num: int) -> None:
        self._worker_num = int(worker_num)
        self._receiver_identities = [b"worker-%d" % r for r in range(self._worker_num)]

    # -- request/gather ----------------------------------------------------------------
    def _send(self, identity: bytes, payload: bytes, deadline: float) -> None:
        while True:
            try:
                self._sock.send_multipart([identity, payload], flags=zmq.NOBLOCK)
                return
            except zmq.ZMQError as e:
                if e.errno not in (zmq.EHOSTUNREACH, zmq.EAGAIN):
                    raise
                if time.monotonic() > deadline:
                    raise ControllerError(f"receiver worker {identity.decode()} is not connected") from None
                time.sleep(0.01)

    def _request(self, messages: list[dict[str, Any]], timeout_s: float | None = None) -> list[dict]:
        """Send one message per worker and gather the replies (ordered like the workers)."""
        if not self._worker_num:
            if self._worker_num == 0:
                return []
            raise ControllerError("set_worker_num() has not been called")
        deadline = time.monotonic() + (timeout_s if timeout_s is not None else self.timeout_s)
        with self._lock:
            rid = next(self._ids)
            for ident, msg in zip(self._receiver_identities, messages):
                self._send(ident, json.dumps(dict(msg, id=rid)).encode(), deadline)
            pending = {ident: None for ident in self._receiver_identities}
            poller = zmq.Poller()
            poller.register(self._sock, zmq.POLLIN)
            while any(v is None for v in pending.values()):
                left = deadline - time.monotonic()
                if left <= 0:
                    missing = [k.decode() for k, v in pending.items() if v is None]
                    raise ControllerError(f"no reply from {missing} within the deadline")
                if not poller.poll(int(min(left, 1.0) * 1000)):
                    continue
                ident, payload = self._sock.recv_multipart()
                reply = json.loads(payload.decode())
                if reply.get("id") != rid or ident not in pending:
                    continue            # late reply to an earlier, timed-out request
                pending[ident] = reply
            return [pending[i] for i in self._receiver_identities]

    def _broadcast(self, msg: dict[str, Any], timeout_s: float | None = None) -> list[dict]:
        return self._request([msg] * (self._worker_num or 0), timeout_s)

    # -- API -----------------------------------------------------------------------------
    def _query_receivers_metadata(self) -> list[dict]:
        """Per-worker ``{"rank", "metadata", "state", ...}``, sorted by rank."""
        replies = self._broadcast({"type": METADATA_REQUEST})
        return sorted(replies, key=lambda r: r.get("rank", -1))

    def get_metadata(self):
        return self._query_receivers_metadata()

    def connect(self, request: ConnectRequest):
        msgs = []
        for idx in range(self._worker_num or 0):
            msgs.append({"type": CONNECT_REQUEST, "master_address": request.master_address,
                         "master_port": request.master_port, "rank": request.base_rank + idx,
                         "world_size": request.world_size, "group_name": request.group_name,
                         "sender_world_size": request.sender_world_size, "backend": request.backend,
                         "session": request.session, "protocol": request.protocol})
        replies = self._request(msgs)
        ok = all(r.get("status") == "ack" for r in replies)
        return {"status": "success" if ok else "error",
                "detail": [r.get("detail") for r in replies if r.get("status") != "ack"]}

    def receive_weights(self):
        replies = self._broadcast({"type": RECEIVE_REQUEST})
        ok = all(r.get("status") == "ack" for r in replies)
        return {"status": "success" if ok else "error",
                "detail": [r.get("detail") for r in replies if r.get("status") != "ack"]}

    def get_stats(self):
        return self._broadcast({"type": STATS_REQUEST})

    def get_metrics(self):
        """Every worker's counters and gauges in the Prometheus text exposition format."""
        from fastapi.responses import PlainTextResponse
        return PlainTextResponse(metrics_text(self.get_stats(), self.prefix),
                                 media_type="text/plain; version=0.0.4")

    def serve(self, host: str = "127.0.0.1", port: int = 0, timeout_s: float = 30.0) -> str:
        """Serve the routes from a uvicorn server on a daemon thread (for rollout processes
        without a FastAPI app of their own); returns the URL the senders use."""
        import socket as _socket
        import uvicorn
        from fastapi import FastAPI
        if port == 0:
            with _socket.socket() as s:
                s.bind((host, 0))
                port = s.getsockname()[1]
        app = FastAPI()
        self.attach(app)
        self._server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="warning"))
        threading.Thread(target=self._server.run, name="wbridge-http", daemon=True).start()
        deadline = time.monotonic() + timeout_s
        while not self._server.started:
            if time.monotonic() > deadline:
                raise ControllerError(f"HTTP server on {host}:{port} did not start within {timeout_s}s")
            time.sleep(0.02)
        return f"http://{host}:{port}{self.prefix}"

    def __enter__(self) -> "WeightReceiverController":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        server = getattr(self, "_server", None)
        if server is not None:
            server.should_exit = True
        self._sock.close(0)
        self._ctx.term()
        try:
            os.unlink(self._ipc_path)
        except OSError:
            pass


_METRICS = (
    ("wbridge_receiver_syncs_total", "counter", "Weight updates the worker completed.",
     lambda w: w.get("totals", {}).get("syncs", 0)),
    ("wbridge_receiver_sync_failures_total", "counter", "Weight updates that failed on the worker.",
     lambda w: w.get("totals", {}).get("failures", 0)),
    ("wbridge_receiver_bytes_total", "counter", "Bytes the worker received.",
     lambda w: w.get("totals", {}).get("bytes", 0)),
    ("wbridge_receiver_epoch", "gauge", "Sync epoch of the worker's current weights.",
     lambda w: w.get("epoch", 0)),
    ("wbridge_receiver_weights_version", "gauge", "Trainer version tag of the current weights (-1: none).",
     lambda w: -1 if w.get("weights_version") is None else w["weights_version"]),
    ("wbridge_receiver_last_update_seconds", "gauge", "Host time of the worker's last update.",
     lambda w: (w.get("syncs") or [{}])[-1].get("host_ms", 0.0) / 1e3),
)


def metrics_text(stats: list[dict], prefix: str = "") -> str:
    """Prometheus exposition text of the workers' ``/wbridge/stats`` replies."""
    extra = f',prefix="{prefix}"' if prefix else ""
    lines = []
    for name, kind, help_, get in _METRICS:
        lines += [f"# HELP {name} {help_}", f"# TYPE {name} {kind}"]
        lines += [f'{name}{{worker="{w.get("rank")}"{extra}}} {get(w)}' for w in stats]
    lines += ["# HELP wbridge_receiver_state Worker state (1 for the current one).",
              "# TYPE wbridge_receiver_state gauge"]
    lines += [f'wbridge_receiver_state{{worker="{w.get("rank")}",state="{w.get("state")}"{extra}}} 1' for w in stats]
    return "\n".join(lines) + "\n"
