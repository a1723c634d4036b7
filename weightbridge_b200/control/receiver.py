"""Rollout-side receiver worker (one per rollout GPU / scheduler process).

A daemon thread serves three ZMQ sockets: a DEALER to the controller (metadata, connect,
receive, stats), a REP for the scheduler's ``request_update`` and, while in a session, a
DEALER bound on TCP through which the first sender arms each sync directly.  State machine:
DISCONNECTED -> CONNECTED (after joining a session) -> AWAITING_SCHEDULER_UPDATE (armed by
``/wbridge/receive`` or by the direct arm message) -> CONNECTED (after the update).

On connect (``gpu_direct``) the worker exports the allocations holding its parameters as
CUDA IPC handles, publishes them with the physical binding of every entry and a flag word
per sender, and checks the senders' plan digests against its own overlap computation.
On update it publishes ``ready/<rank>/<epoch>``; the senders' kernels store straight into
the parameters and write the epoch to the flags; the worker waits (bounded) for every
expected sender's ``done`` key, then reads the flag words back (one small device->host
copy) and accepts the update only if every flag holds this epoch.

Parity: ``wbridge/frontend/receiver.py:48-230``.  Differences: ``stop()`` stops the thread,
the thread is a daemon, every wait has a deadline, the handshake only involves senders
that overlap this worker (the reference waits on every sender), the state_dict is bound at
connect (the senders write into it directly), and ``request_update`` can wait for arming.
"""
from __future__ import annotations

import json
import logging
import os
import socket
import tempfile
import threading
import time
import uuid
from collections import deque
from typing import Any

import torch
import zmq

from ..core.binding import bind
from ..core.plan import lower_ops, phys_binding, plan_digest, plan_pair
from ..core.shard import WeightData
from ..utils.config import WIRE_MODES, TransferConfig, normalize_mode
from ..utils.trace import nvtx_range
from .assign import expected_senders, restrict
from .protocol import (CONNECT_REQUEST, METADATA_REQUEST, PROTOCOL_VERSION, RECEIVE_REQUEST, STATS_REQUEST,
                       STOP_REQUEST, UPDATE_REQUEST, ReceiverState, b64, gpu_id)
from .session import Janitor, PeerError, Session, SessionTimeout
from .board import word_digest

logger = logging.getLogger(__name__)


class ReceiveError(RuntimeError):
    pass


class WeightReceiver:
    """One rollout worker's side of the weight sync (one per GPU worker process).

    ``controller_ipc_name``: ``WeightReceiverController.ipc_name`` of the rollout server;
    ``rank``: the worker's index among the controller's ``worker_num`` workers;
    ``metadata``: the worker's shards as logical HF boxes; ``state_dict``: the tensors (or
    views into fused parameters) the senders write into, bound at connect, or ``None`` to
    hand them over at the first ``request_update``; ``device`` defaults to the tensors'.
    The scheduler calls ``request_update(timeout=...)`` between batches.
    """

    def __init__(self, controller_ipc_name: str, rank: int, metadata: WeightData,
                 state_dict: dict[str, Any] | None = None, device: torch.device | int | str | None = None,
                 config: TransferConfig | None = None):
        self.controller_ipc_name = controller_ipc_name
        self.rank = rank
        self.metadata = metadata if isinstance(metadata, WeightData) else WeightData(metadata)
        self.state_dict = state_dict
        self.config = config or TransferConfig.from_env()
        self.device = self._infer_device(device, state_dict)
        self._state = ReceiverState.DISCONNECTED
        self._error: str | None = None
        self._stop = threading.Event()
        self._started = threading.Event()
        self.stats: deque = deque(maxlen=64)
        self.totals = {"syncs": 0, "failures": 0, "bytes": 0}     # since construction (metrics counters)
        self.epoch = 0
        self.weights_version: int | None = None       # the tag of the last weights received (send(version=))
        self.session: Session | None = None
        self._pending_update: dict | None = None
        self._garbage: list[str] = []
        self._arm_sock = None
        self._poller: zmq.Poller | None = None
        self._janitor: Janitor | None = None
        self._watch = None
        self._bind_gen = 0                            # bumped at every (re)binding of the tensors
        self._rebind_to = None                        # tensors handed to rebind(), bound at the next update
        self._rebind_lock = threading.Lock()
        self._bound = False                           # tensors bound and exported for this session
        self._pull_versions, self._pull_prog, self._pull_imports = None, None, {}   # pull direction
        self._pull_devices: dict[int, int] = {}      # GPU ordinal of each sender pulled from
        self._gpu_id: str | None | bool = False       # this worker's GPU UUID (False: not read yet)
        self._pull_stream = None
        self._pull_progs: dict = {}                   # pull programs by entry-subset digest
        self._pull_src: dict = {}
        self._pull_ranges: list = []
        self._mc = None                               # nvls: (multicast object, replica group)
        self._board = None                            # same-host handshake words (control/board.py)
        self._pull_phases: dict = {}                  # host time of the last pull's steps, ms
        self._arm_t = 0.0                             # time.perf_counter() of the last direct arm
        self._pulled_t = 0.0                          # ... and of the last pulled word
        self._arm_path = None                         # Unix socket file of a loopback arm endpoint
        self._fd_server = None                        # nvls: serves the pool's file descriptor
        fd, path = tempfile.mkstemp(prefix=f"wbridge_sched_{rank}_")
        os.close(fd)
        os.unlink(path)
        self._sched_path = path
        self.scheduler_ipc_name = f"ipc://{path}"
        self._ctx = zmq.Context()
        self.receiver_thread = threading.Thread(target=self._loop, name=f"wbridge-receiver-{rank}", daemon=True)
        self.receiver_thread.start()
        if not self._started.wait(30):
            raise ReceiveError("receiver thread did not start")
        self._req_lock = threading.Lock()
        self._req = self._new_req()

    @staticmethod
    def _infer_device(device, state_dict) -> torch.device:
        if device is not None:
            return torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if state_dict:
            for v in state_dict.values():
                t = v[0] if isinstance(v, (list, tuple)) else v
                if isinstance(t, torch.Tensor):
                    return t.device
        if torch.cuda.is_available():
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")

    def _new_req(self):
        s = self._ctx.socket(zmq.REQ)
        s.setsockopt(zmq.LINGER, 0)
        s.setsockopt(zmq.REQ_RELAXED, 1)
        s.setsockopt(zmq.REQ_CORRELATE, 1)
        s.connect(self.scheduler_ipc_name)
        return s

    @property
    def state(self) -> ReceiverState:
        return self._state

    def set_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Tensors (or views) the senders write into; bound at the next connect."""
        self.state_dict = state_dict
        self.device = self._infer_device(None, state_dict)

    def rebind(self, state_dict: dict[str, Any]) -> None:
        """Receive into other tensors from the next update on (the engine reallocated its
        parameters): the worker binds and exports them at that update and the senders pick
        the new memory up when they see its ready key, without a reconnect."""
        if self.mode == "nvls":
            raise ReceiveError("rebind is not supported in mode 'nvls' (its memory is a fixed VmmPool)")
        with self._rebind_lock:
            self._rebind_to = state_dict

    # -- scheduler side ----------------------------------------------------------------
    def request_update(self, state_dict: dict[str, Any] | None = None, timeout: float | None = None) -> bool:
        """Receive the pending weights into the bound state_dict.

        Returns False when no sync is pending (the controller has not armed this worker);
        with ``timeout`` the call first waits up to that many seconds for the arm.  A sync
        that started and then failed (a sender's error, a stale flag, a deadline) raises
        ``ReceiveError`` instead of returning False: the parameters may hold a mix of old and
        new values, which the caller must not mistake for "no update".
        """
        if state_dict is not None and state_dict is not self.state_dict:
            if self._bound:
                if not self._same_tensors(state_dict):
                    raise ReceiveError("request_update got tensors other than the ones bound at connect; "
                                       "reconnect the sender to rebind")
            else:
                self.set_state_dict(state_dict)
        msg = {"type": UPDATE_REQUEST, "wait_s": float(timeout or 0.0)}
        wait = (timeout or 0.0) + self.config.sync_timeout_s + 5.0
        with self._req_lock:
            self._req.send_string(json.dumps(msg))
            if not self._req.poll(int(wait * 1000)):
                self._req.close(0)
                self._req = self._new_req()
                raise ReceiveError(f"no reply from the receiver thread within {wait:.0f}s")
            reply = json.loads(self._req.recv_string())
        if reply.get("error"):
            raise ReceiveError(reply["error"])
        return bool(reply["success"])

    def wait_for_version(self, version: int, timeout: float, poll_s: float = 1.0) -> int:
        """Take pending updates until the weights carry at least trainer version ``version``
        (``send(version=...)``); returns the version reached.  For a scheduler that must not
        generate with weights older than a given step.  Raises ``ReceiveError`` when the
        deadline passes first (or an update fails)."""
        deadline = time.monotonic() + timeout
        while self.weights_version is None or self.weights_version < version:
            left = deadline - time.monotonic()
            if left <= 0:
                raise ReceiveError(f"weights still at version {self.weights_version} after {timeout:.1f}s "
                                   f"(waiting for {version})")
            self.request_update(timeout=min(poll_s, left))
        return self.weights_version

    def _same_tensors(self, state_dict) -> bool:
        for name in self.metadata.names():
            a, b = self.state_dict.get(name), state_dict.get(name)
            if isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor) and a.data_ptr() != b.data_ptr():
                return False
        return True

    def __enter__(self) -> "WeightReceiver":
        return self

    def __exit__(self, *exc) -> None:
        self.stop()

    def stop(self) -> None:
        """Stop the worker thread and release the session."""
        self._stop.set()
        if self.receiver_thread.is_alive():
            # a pool bound to a multicast object is unbound by the worker thread once the
            # senders unmapped it (bounded wait): the process must not exit before that
            self.receiver_thread.join(timeout=10 if self._mc is None else self.config.connect_timeout_s + 30)
        try:
            self._req.close(0)
        except Exception:
            pass
        self._ctx.term()
        for p in (self._sched_path,):
            try:
                os.unlink(p)
            except OSError:
                pass

    # -- worker thread -----------------------------------------------------------------
    def _loop(self) -> None:
        ctl = self._ctx.socket(zmq.DEALER)
        ctl.setsockopt(zmq.IDENTITY, f"worker-{self.rank}".encode())
        ctl.setsockopt(zmq.LINGER, 0)
        ctl.connect(self.controller_ipc_name)
        rep = self._ctx.socket(zmq.REP)
        rep.setsockopt(zmq.LINGER, 0)
        rep.bind(self.scheduler_ipc_name)
        poller = zmq.Poller()
        poller.register(ctl, zmq.POLLIN)
        poller.register(rep, zmq.POLLIN)
        self._poller = poller
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        self._started.set()
        try:
            while not self._stop.is_set():
                socks = dict(poller.poll(50))
                if ctl in socks:
                    data = json.loads(ctl.recv_string())
                    self._on_controller(ctl, data)
                arm = self._arm_sock
                if arm is not None and arm in socks:
                    self._on_arm(json.loads(arm.recv_string()))
                if rep in socks:
                    msg = json.loads(rep.recv_string())
                    self._on_scheduler(rep, msg)
                if self._pending_update is not None:
                    self._try_pending(rep)
        finally:
            ctl.close(0)
            rep.close(0)
            self._teardown()

    def _reply(self, sock, data: dict, obj: dict) -> None:
        obj = dict(obj, id=data.get("id"))
        sock.send_string(json.dumps(obj))

    def _on_controller(self, sock, data: dict) -> None:
        t = data.get("type")
        if t == METADATA_REQUEST:
            if self._gpu_id is False:
                self._gpu_id = gpu_id(self.device)
            self._reply(sock, data, {"rank": self.rank, "metadata": self.metadata.to_jsonable(),
                                     "state": self._state.value, "device": str(self.device),
                                     "gpu": self._gpu_id, "host": socket.gethostname(), "pid": os.getpid()})
        elif t == CONNECT_REQUEST:
            if self._state == ReceiverState.AWAITING_SCHEDULER_UPDATE:
                self._reply(sock, data, {"status": "error", "detail": "cannot connect while awaiting scheduler update"})
                return
            if int(data.get("protocol", 1)) != PROTOCOL_VERSION:
                self._reply(sock, data, {"status": "error", "detail": f"sender speaks protocol {data.get('protocol', 1)}, "
                                                                      f"this receiver {PROTOCOL_VERSION}"})
                return
            self._reply(sock, data, {"status": "ack"})
            self._state = ReceiverState.CONNECTING
            try:
                self._join(data)
                self._state = ReceiverState.CONNECTED
                self._error = None
            except Exception as e:  # published to the session so the senders fail fast
                logger.exception("receiver %d failed to join", self.rank)
                self._error = f"{type(e).__name__}: {e}"
                self._state = ReceiverState.FAILED
                if self.session is not None:
                    gr = data["rank"]
                    self.session.set_error([f"recv/{gr}", f"verified/{gr}", f"joined/{gr}"],
                                           f"receiver {gr}: {self._error}")
        elif t == RECEIVE_REQUEST:
            if self._state != ReceiverState.CONNECTED:
                self._reply(sock, data, {"status": "error", "detail": f"requires CONNECTED state, is {self._state.value}"})
                return
            self._state = ReceiverState.AWAITING_SCHEDULER_UPDATE
            self._reply(sock, data, {"status": "ack"})
        elif t == STATS_REQUEST:
            self._reply(sock, data, {"rank": self.rank, "state": self._state.value, "epoch": self.epoch,
                                     "weights_version": self.weights_version, "error": self._error,
                                     "syncs": list(self.stats), "totals": dict(self.totals)})
        elif t == STOP_REQUEST:
            self._reply(sock, data, {"status": "ack"})
            self._stop.set()
        else:
            self._reply(sock, data, {"status": "error", "detail": f"unknown message type {t!r}"})

    def _on_arm(self, msg: dict) -> None:
        """A sender armed sync ``epoch`` directly (same transition as ``/wbridge/receive``).
        A worker that cannot take it writes the reason into its ready key, where every
        sender of the session is waiting."""
        if "epoch" not in msg or self.session is None:
            return                                   # connection probe
        epoch = int(msg["epoch"])
        ok_states = (ReceiverState.CONNECTED, ReceiverState.AWAITING_SCHEDULER_UPDATE)   # re-arm: no-op
        if self._state in ok_states and epoch == self.epoch + 1:
            self._state = ReceiverState.AWAITING_SCHEDULER_UPDATE
            self._arm_t = time.perf_counter()
            return
        why = (f"receiver {self.global_rank} cannot take sync {epoch}: state {self._state.value}, "
               f"last epoch {self.epoch}")
        # senders wait for ready (push) or pulled (pull): both carry the reason
        self.session.set_error([f"ready/{self.global_rank}/{epoch}", f"pulled/{self.global_rank}/{epoch}"], why)

    def _open_arm_socket(self, master_address: str) -> str:
        """Bind the direct-arm DEALER; returns its endpoint.  With a loopback session (every
        sender on this host) a Unix-domain socket, which delivers an arm in about half the time
        of a TCP loopback connection; otherwise an OS-chosen TCP port."""
        from .session import host_address
        loopback = master_address in ("127.0.0.1", "localhost", "::1")
        sock = self._ctx.socket(zmq.DEALER)
        sock.setsockopt(zmq.LINGER, 0)
        sock.setsockopt(zmq.IDENTITY, f"wbarm-{self.global_rank}".encode())
        self._arm_sock = sock
        self._poller.register(sock, zmq.POLLIN)
        if loopback:
            self._arm_path = os.path.join(tempfile.gettempdir(), f"wbridge-arm-{os.getpid()}-{uuid.uuid4().hex[:12]}")
            endpoint = f"ipc://{self._arm_path}"
            sock.bind(endpoint)
            return endpoint
        port = sock.bind_to_random_port("tcp://*")
        return f"tcp://{host_address()}:{port}"

    def _open_watch(self, master_address: str):
        """Accept the senders' liveness connections (``control/liveness.py``)."""
        from .liveness import PeerWatch
        from .session import host_address
        loopback = master_address in ("127.0.0.1", "localhost", "::1")
        lsock, port = PeerWatch.listen("127.0.0.1" if loopback else "0.0.0.0")
        self._live_addr = ["127.0.0.1" if loopback else host_address(), port]
        return PeerWatch(self._sender_lost, lsock)

    def _sender_lost(self, s: int) -> None:
        """A sender's process is gone: fail the wait for its ``done`` key now, not at the deadline."""
        janitor, gr = self._janitor, self.global_rank
        if janitor is not None and s in getattr(self, "expected", []):
            janitor.set_error([f"done/{s}/{gr}/{self.epoch + 1}"],
                              f"sender {s} left the session (its connection to receiver {gr} closed)")

    def _close_arm_socket(self) -> None:
        sock, self._arm_sock = self._arm_sock, None
        if sock is not None:
            try:
                self._poller.unregister(sock)
            except KeyError:
                pass
            sock.close(0)
        path, self._arm_path = self._arm_path, None
        if path:
            try:
                os.unlink(path)
            except OSError:
                pass

    def _on_scheduler(self, sock, msg: dict) -> None:
        if msg.get("type") != UPDATE_REQUEST:
            sock.send_string(json.dumps({"success": False, "message": "unknown message"}))
            return
        if self._state == ReceiverState.AWAITING_SCHEDULER_UPDATE:
            self._do_update(sock)
            return
        wait_s = float(msg.get("wait_s") or 0.0)
        if wait_s > 0 and self._state in (ReceiverState.CONNECTED, ReceiverState.CONNECTING,
                                          ReceiverState.DISCONNECTED):
            self._pending_update = {"deadline": time.monotonic() + wait_s}
            return
        sock.send_string(json.dumps({"success": False, "message": "no pending weights",
                                     "state": self._state.value}))

    def _try_pending(self, sock) -> None:
        if self._state == ReceiverState.AWAITING_SCHEDULER_UPDATE:
            self._pending_update = None
            self._do_update(sock)
        elif time.monotonic() > self._pending_update["deadline"]:
            self._pending_update = None
            sock.send_string(json.dumps({"success": False, "message": "no pending weights"}))

    def _do_update(self, sock) -> None:
        try:
            with nvtx_range("wbridge.receive"):
                rec = self._receive()
            self.stats.append(rec)
            self.totals["syncs"] += 1
            self.totals["bytes"] += int(rec.get("bytes") or 0)
            self._state = ReceiverState.CONNECTED
            sock.send_string(json.dumps({"success": True, "epoch": self.epoch, "stats": rec}))
            self._collect_garbage()
        except Exception as e:
            logger.exception("receiver %d update failed", self.rank)
            self.totals["failures"] += 1
            self._error = f"{type(e).__name__}: {e}"
            self._state = ReceiverState.FAILED
            if self._janitor is not None:        # off this thread: the store may be gone with its host
                self._janitor.set_error([f"ready/{self.global_rank}/{self.epoch + 1}"],
                                        f"receiver {self.global_rank}: {self._error}")
            sock.send_string(json.dumps({"success": False, "message": self._error, "error": self._error}))

    # -- session -----------------------------------------------------------------------
    def _join(self, data: dict) -> None:
        self._teardown()
        mode = normalize_mode(data["backend"])
        self.mode = mode
        gr = int(data["rank"])
        self.global_rank = gr
        W = int(data["sender_world_size"])
        self.world_size = int(data["world_size"])
        sess = Session(data["master_address"], int(data["master_port"]), is_master=False,
                       timeout_s=self.config.connect_timeout_s)
        self.session = sess
        self._janitor = Janitor(data["master_address"], int(data["master_port"]), self.config.connect_timeout_s)
        self._watch = self._open_watch(data["master_address"])
        info: dict[str, Any] = {"rank": gr, "worker": self.rank, "pid": os.getpid(), "host": socket.gethostname(),
                                "mode": mode, "arm": self._open_arm_socket(data["master_address"]),
                                "live": self._live_addr}
        self._W = W
        self._bound = False
        if self.state_dict is not None:
            info.update(self._bind())
        elif mode == "nvls":
            raise ReceiveError("mode 'nvls' needs the receiver's state_dict (inside a VmmPool) before connect")
        else:
            # late binding: the tensors arrive with the first request_update(state_dict)
            info["late"] = True
        sess.set_json(f"recv/{gr}", info)
        # plan agreement: recompute every expected sender's overlap and compare digests
        assignment = sess.get_json("assign")
        smetas = sess.get_json("senders/meta")
        plan = {int(s): {int(r): v for r, v in rs.items()} for s, rs in assignment.items()}
        self.expected = expected_senders(plan, gr)
        self._names = {s: plan[s][gr] for s in self.expected}
        self.direction = sess.wait_checked(["direction"])[0].decode() if mode == "gpu_direct" else "push"
        if mode in ("gpu_direct", "nvls"):
            from .board import SyncBoard
            self._board = SyncBoard.attach(sess.get_json("board", self.config.connect_timeout_s))
        self._wire_chunk = int(sess.wait_checked(["wire_chunk"])[0]) if mode in WIRE_MODES else 0
        self._pull_versions, self._pull_prog, self._pull_imports = None, None, {}
        self.expected_bytes = 0
        self.overlaps: dict[int, WeightData] = {}
        for s in self.expected:
            ov = WeightData.compute_overlap(restrict(WeightData(smetas[s]), plan[s][gr]), self.metadata)
            digest = sess.wait_checked([f"digest/{s}/{gr}"])[0].decode()
            if digest != plan_digest(ov):
                raise ReceiveError(f"plan digest mismatch with sender {s}: the two sides disagree on the layout")
            self.overlaps[s] = ov
            self.expected_bytes += ov.total_nbytes()
        sess.set(f"verified/{gr}", "1")
        if mode == "nvls" and self.device.type == "cuda":
            self._join_nvls_group(sess, gr)
        if mode in WIRE_MODES:
            from .sender import wire_group
            self._pg = wire_group(mode, sess, gr, self.world_size, self.config.connect_timeout_s,
                                  data["master_address"])
            self._wires = None
            if self._bound:
                self._setup_wires()
        self.epoch = 0
        sess.set(f"joined/{gr}", "1")
        logger.info("receiver worker %d joined session as rank %d (mode=%s, senders=%s, %.3f GB expected)",
                    self.rank, gr, mode, self.expected, self.expected_bytes / 1e9)

    def _bind(self) -> dict:
        """Bind the state_dict to the metadata and describe the memory for the senders."""
        mode, W = self.mode, self._W
        binding = bind(self.metadata, self.state_dict)
        self._rphys_abs = phys_binding(binding)          # local addresses (pull programs write here)
        info: dict[str, Any] = {}
        if mode in ("gpu_direct", "nvls") and self.device.type == "cpu":
            # host memory: only a sender in this same process can write it (tests, CPU runs)
            self.flags = torch.zeros(max(W, 1), dtype=torch.int64)
            phys = phys_binding(binding)
            info.update({"device": -1, "allocs": [], "binding": phys.to_json(),
                         "flags": [-1, self.flags.data_ptr(), W]})
        elif mode == "nvls":
            self._join_nvls_export(binding, info, W)
        elif mode == "gpu_direct":
            from ..parallel.ipc import ExportTable
            from ..ops._ext import ext
            torch.cuda.set_device(self.device)
            self.flags = torch.zeros(max(W, 1), dtype=torch.int64, device=self.device)
            export = ExportTable(self.device)
            phys = phys_binding(binding, export.locate)
            falloc, foff = export.locate(self.flags.data_ptr())
            info.update({"device": self.device.index, "uuid": b64(ext().device_uuid(self.device.index)),
                         "allocs": export.to_json(), "binding": phys.to_json(), "flags": [falloc, foff, W]})
            self._export = export
        else:
            self._rphys = phys_binding(binding)
        self._bound = True
        self._bind_gen += 1
        info["gen"] = self._bind_gen
        return info

    def _setup_wires(self) -> None:
        """Wire modes: per expected sender, the chunked receive buffers and unpack tables
        (``control/wires.py``)."""
        from ..core.plan import storage_ranges
        from .wires import WireSet
        if (self.mode == "nccl") != (self.device.type == "cuda"):
            raise ReceiveError(f"mode {self.mode} does not take tensors on {self.device}")
        self._wires = WireSet.for_receiver(self._rphys, self.overlaps, self.device, self.config,
                                           storage_ranges(self.state_dict.values()), self._wire_chunk)
        self._wire_sets = {"": self._wires}        # by the digest of a partial sync's entry subset
        if self.device.type == "cuda":
            self._stream = torch.cuda.Stream(self.device)

    def _wire_set(self, digest: str):
        """The wire set of the entry subset ``digest`` names (``""``: every entry), cut like
        the senders' from the same overlaps and on the full set's buffers."""
        ws = self._wire_sets.get(digest)
        if ws is None:
            from ..core.plan import storage_ranges
            from ..core.wire import restrict_overlap
            from .wires import WireSet
            names = self.session.get_json(f"subset/{digest}", self.config.sync_timeout_s)
            overlaps = {s: restrict_overlap(ov, names) for s, ov in self.overlaps.items()}
            ws = WireSet.for_receiver(self._rphys, overlaps, self.device, self.config,
                                      storage_ranges(self.state_dict.values()), self._wire_chunk,
                                      self._wire_sets[""].buffers())
            if len(self._wire_sets) >= 8:
                self._wire_sets.pop(next(k for k in self._wire_sets if k))
            self._wire_sets[digest] = ws
        return ws

    def _late_bind(self) -> None:
        """First update of a receiver that joined without tensors: bind, export, publish."""
        if self.state_dict is None:
            raise ReceiveError("request_update needs the state_dict to receive into")
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        extra = self._bind()
        self._pull_versions = None                # the pull program writes into the old tensors
        if self.mode in WIRE_MODES:
            self._setup_wires()
        else:
            self.session.set_json(f"recvbind/{self.global_rank}", extra)

    def _receive(self) -> dict:
        sess = self.session
        if sess is None:
            raise ReceiveError("not connected")
        epoch = self.epoch + 1
        gr = self.global_rank
        t0 = time.perf_counter()
        with self._rebind_lock:
            target, self._rebind_to = self._rebind_to, None
        if target is not None:
            self.set_state_dict(target)
            self._bound = False
        if not self._bound:
            self._late_bind()
        if self.device.type == "cuda":
            # the engine's last batch may still be running on its streams, reading these
            # parameters: only an idle device may be written by the senders
            torch.cuda.synchronize(self.device)
        phases: dict[str, float] = {}             # host time of this update's steps, ms
        mark = [t0]

        def lap(name: str) -> None:
            t = time.perf_counter()
            phases[name] = round((t - mark[0]) * 1e3, 4)
            mark[0] = t

        lap("idle")
        if self.mode in WIRE_MODES:
            try:     # sender rank 0 writes the tag and the entry subset before it arms the workers
                tag, _sep, digest = sess.wait_checked([f"ver/{epoch}"], self.config.sync_timeout_s)[0] \
                    .decode().partition("|")
                ws = self._wire_set(digest)
            except (SessionTimeout, PeerError) as e:
                raise ReceiveError(str(e)) from None
            version = int(tag)
            sess.set(f"ready/{gr}/{epoch}", "1")
            if ws.device.type == "cuda":     # NCCL receives and unpack launches, ordered on one stream
                with torch.cuda.stream(self._stream):
                    ws.recv(self._pg, epoch, self._stream)
                self._stream.synchronize()
            else:
                ws.recv(self._pg, epoch)
        else:
            b = self._board
            keys = [f"done/{s}/{gr}/{epoch}" for s in self.expected]
            what = f"senders {self.expected} to finish epoch {epoch}"
            try:
                if b is not None:
                    b.publish(b.ready_slot(gr), [self._bind_gen], epoch)          # senders rebind on a new generation
                    b.wait([b.done_slot(s, gr) for s in self.expected], epoch, self.config.sync_timeout_s,
                           lambda: sess.raise_posted_error(keys), what)
                    lap("ready")
                    words = [b.read(b.done_slot(s, gr), 6) for s in self.expected]
                    done = [[str(w[1]), str(w[2]), str(w[3]), str(w[4]), word_digest(w[5])] for w in words]
                else:
                    sess.set(f"ready/{gr}/{epoch}", str(self._bind_gen))
                    vals = sess.wait_checked(keys, self.config.sync_timeout_s, what=what)
                    done = [v.decode().split(":") for v in vals]          # status:binding-version:pushed:tag:subset
            except (SessionTimeout, PeerError) as e:
                raise ReceiveError(str(e)) from None
            bad = {s: int(d[0]) for s, d in zip(self.expected, done) if int(d[0])}
            if bad:
                raise ReceiveError(f"senders reported kernel status {bad} for epoch {epoch}")
            pushed = [s for s, d in zip(self.expected, done) if len(d) < 3 or d[2] == "1"]
            version = max((int(d[3]) for d in done if len(d) > 3), default=-1)
            lap("done")
            if self.direction == "pull":
                self._pull(epoch, {s: int(d[1]) for s, d in zip(self.expected, done)},
                           done[0][4] if done and len(done[0]) > 4 else "")
                lap("pull")
                phases.update(self._pull_phases)
            if self.config.verify_flags and pushed:
                flags = self.flags.cpu()
                stale = [s for s in pushed if int(flags[s]) != epoch]
                if stale:
                    raise ReceiveError(f"flags of senders {stale} do not hold epoch {epoch}: {flags.tolist()}")
            # handshake keys of this epoch are deleted after the reply (off the critical path)
            if b is None:
                self._garbage += [f"done/{s}/{gr}/{epoch}" for s in self.expected]
                if epoch > 1:
                    self._garbage.append(f"ready/{gr}/{epoch - 1}")
        self.epoch = epoch
        self.weights_version = None if version < 0 else version
        lap("finish")
        return {"epoch": epoch, "version": self.weights_version, "host_ms": (time.perf_counter() - t0) * 1e3,
                "bytes": self.expected_bytes, "senders": self.expected, "phases_ms": phases,
                "marks": {"armed": self._arm_t, "begin": t0, "pulled": self._pulled_t, "end": mark[0]}}

    # -- pull direction --------------------------------------------------------------------
    def _pull(self, epoch: int, versions: dict[int, int], digest: str = "") -> None:
        """Load this worker's copies from the senders' memory (they keep it unchanged until
        every receiver has reported ``pulled``); ``digest`` names a partial sync's entries."""
        status = 0
        try:
            self._select_pull(versions, digest)
            prog = self._pull_prog
            if prog is not None and len(prog.tables):
                if prog.device.type == "cpu":
                    prog.launch(epoch, signal=False)
                else:
                    # the epoch goes down from pinned memory with the launch; the kernel's last
                    # CTA publishes it to this worker's pull flag, read back with the status
                    with nvtx_range("wbridge.receive/pull"):
                        t0 = time.perf_counter()
                        prog.launch(epoch, self._pull_stream, signal=True)
                        t1 = time.perf_counter()
                        self._pull_stream.synchronize()
                        t2 = time.perf_counter()
                    status, got = prog.read_status_and_flag()
                    self._pull_phases = {"pull_enqueue": round((t1 - t0) * 1e3, 4),
                                         "pull_device_wait": round((t2 - t1) * 1e3, 4),
                                         "pull_readback": round((time.perf_counter() - t2) * 1e3, 4)}
                    if not status and got != epoch:
                        raise ReceiveError(f"pull kernel completed with flag {got}, expected epoch {epoch}")
        except Exception as e:
            self.session.set_error([f"pulled/{self.global_rank}/{epoch}"], f"receiver {self.global_rank}: {e}")
            raise
        if self._board is not None:
            self._board.publish(self._board.pulled_slot(self.global_rank), [status], epoch)
            self._pulled_t = time.perf_counter()
        else:
            self.session.set(f"pulled/{self.global_rank}/{epoch}", str(status))
            if epoch > 1:   # the senders read epoch e's key before this worker can reach epoch e + 1
                self._garbage.append(f"pulled/{self.global_rank}/{epoch - 1}")
        if status:
            raise ReceiveError(f"pull kernel reported status {status:#x} at epoch {epoch}")

    def _select_pull(self, versions: dict[int, int], digest: str) -> None:
        """Make the pull program of (the senders' memory versions, entry subset) current: the
        senders' memory is opened again when a version changes, a subset's program is compiled
        on first use."""
        if versions != self._pull_versions:
            self._open_senders(versions)
        prog = self._pull_progs.get(digest)
        if prog is None:
            names = set(self.session.get_json(f"subset/{digest}", self.config.sync_timeout_s)) if digest else None
            prog = self._compile_pull(names)
            if len(self._pull_progs) >= 8:
                self._pull_progs.pop(next(k for k in self._pull_progs if k))
            self._pull_progs[digest] = prog
        self._pull_prog = prog

    def _open_senders(self, versions: dict[int, int]) -> None:
        from ..core.plan import PhysBinding
        from ..parallel.ipc import ImportTable
        from .sender import _phys_extents
        for imp in self._pull_imports.values():
            imp.close()
        self._pull_imports, self._pull_src, self._pull_ranges = {}, {}, []
        self._pull_devices = {}
        self._pull_progs = {}
        for s in self.expected:
            sb = self.session.get_json(f"sendbind/{s}", self.config.sync_timeout_s)
            if sb["host"] != socket.gethostname():
                raise ReceiveError(f"sender {s} is on host {sb['host']}: pulling needs one node")
            same = sb["pid"] == os.getpid()
            if not sb["allocs"] and not same:
                raise ReceiveError(f"sender {s} holds host memory in another process")
            imp = ImportTable(sb["allocs"], same_process=same)
            self._pull_imports[s] = imp
            self._pull_devices[s] = int(sb.get("device", -1))
            sphys = PhysBinding.from_json(sb["binding"])
            self._pull_src[s] = sphys
            if sb["allocs"]:
                self._pull_ranges += [(imp.base(i), imp.base(i) + int(a["size"])) for i, a in enumerate(sb["allocs"])]
            else:
                self._pull_ranges += _phys_extents(sphys)
        self._pull_versions = dict(versions)
        if self.device.type != "cpu" and self._pull_stream is None:
            self._pull_stream = torch.cuda.Stream(self.device)

    def _compile_pull(self, names: set | None):
        """The pull program of every expected sender's entries (restricted to ``names``)."""
        from ..core.plan import storage_ranges, validate_tables
        from ..ops.executor import HostProgram, LaunchConfig, TransferProgram
        from .sender import _interleave
        parts, routes = [], []
        me = self.device.index if self.device.type == "cuda" else -1
        for s in self.expected:
            mine = self._names[s] if names is None else [n for n in self._names[s] if n in names]
            ops = [o for o in plan_pair(self._pull_src[s], self._rphys_abs, names=mine)
                   if o.kind not in ("quant", "squant")]
            parts.append(lower_ops(ops, self._pull_imports[s].base, lambda a: 0, item_bytes=self.config.item_bytes))
            if parts[-1].bytes_written:
                routes.append({"src": self._pull_devices.get(s, -1), "dst": [me], "bytes": int(parts[-1].bytes_written),
                               "multicast": False})
        # round-robin over the senders, so the CTAs running at any moment load from every
        # sender at once (one sender after the other would leave all but one egress idle)
        tables = _interleave(parts)
        if self.config.validate_plan:
            validate_tables(tables, self._pull_ranges, storage_ranges(self.state_dict.values()))
        if self.device.type == "cpu":
            prog = HostProgram(tables)
        else:
            prog = TransferProgram(tables, self.device, [], LaunchConfig(mode=self.config.kernel_mode), local_flag=True)
        prog.routes = routes
        return prog

    def launch(self, stream: torch.cuda.Stream | None = None) -> None:
        """Pull direction: enqueue this worker's pull kernel on ``stream`` with no handshake
        (for callers that know the senders' memory is stable, e.g. device-timed benchmarks).
        Needs one completed ``request_update`` (which compiles the pull program)."""
        prog = self._pull_prog
        if prog is None:
            raise RuntimeError("no pull program: the receiver is not in the pull direction or has not synced yet")
        if len(prog.tables):
            if prog.device.type == "cpu":
                prog.launch(0, signal=False)
            else:
                prog.launch(0, stream or torch.cuda.current_stream(prog.device), signal=False)

    @property
    def pull_program(self):
        return self._pull_prog

    def routes(self) -> list[dict]:
        """Where the current pull program's bytes come from: one record per sender, with the
        GPU ordinals on both ends."""
        return list(getattr(self._pull_prog, "routes", [])) if self._pull_prog is not None else []

    # -- NVLink multicast (mode "nvls") -----------------------------------------------------
    def _join_nvls_export(self, binding, info: dict, W: int) -> None:
        """Publish this worker's VMM pool (file descriptor server) and its pool-relative binding."""
        from ..ops._ext import ext
        from ..parallel.fdpass import FdServer
        from ..parallel.vmm import find_pool
        torch.cuda.set_device(self.device)
        pools = {id(find_pool(bs.tensor.data_ptr())) for views in binding.entries.values() for bs in views}
        pool = find_pool(next(iter(binding.entries.values()))[0].tensor.data_ptr()) if binding.entries else None
        if pool is None or len(pools) != 1:
            raise ReceiveError("mode 'nvls' needs every bound parameter inside one VmmPool "
                               "(weightbridge_b200.parallel.vmm.VmmPool)")
        self._pool = pool
        self.flags = pool.tail(8 * max(W, 1)).view(torch.int64)
        self.flags.zero_()
        phys = phys_binding(binding, lambda ptr: (0, ptr - pool.ptr))
        self._fd_server = FdServer()
        self._fd_server.publish("pool", pool.export_fd())
        info.update({"device": self.device.index, "uuid": b64(ext().device_uuid(self.device.index)),
                     "allocs": [{"vmm": True, "fd_addr": self._fd_server.address, "key": "pool",
                                 "size": pool.size, "base": pool.ptr}],
                     "binding": phys.to_json(), "flags": [0, self.flags.data_ptr() - pool.ptr, W],
                     "pool": {"size": pool.size}})

    def _join_nvls_group(self, sess, gr: int) -> None:
        """Join this worker's replica group: add the device, bind the pool (see parallel/nvls.py)."""
        from ..parallel.nvls import McMember
        plan = sess.get_json("nvls/plan", self.config.connect_timeout_s)
        self._mc = None
        for g in plan["groups"]:
            if gr not in g["replicas"]:
                continue
            m = McMember(g["id"], g["size"], self.device.index)
            self._mc = (m, g)                 # tracked from here on: teardown undoes every stage
            m.join(g["addr"])
            m.add_device()
            everyone = g["replicas"] + g["senders"]
            sess.set(f"nvls/{g['id']}/added/{gr}", "1")
            sess.wait_checked([f"nvls/{g['id']}/added/{x}" for x in everyone], self.config.connect_timeout_s,
                              "multicast members to add their devices")
            m.bind(self._pool)
            sess.set(f"nvls/{g['id']}/bound/{gr}", "1")

    def _leave_nvls(self) -> None:
        """Unbind only once every sender of the group unmapped the object (bounded wait)."""
        mc = self._mc
        if not mc:
            return
        m, g = mc
        try:
            if self.session is not None:
                self.session.wait([f"nvls/{g['id']}/unmapped/{x}" for x in g["senders"]],
                                  self.config.connect_timeout_s, "senders to unmap the multicast object")
        except SessionTimeout as e:
            # the store lives in sender rank 0, which closes it only after every sender of every
            # group it created reported the unmap (or its own bounded wait for that ended)
            logger.warning("receiver %d: multicast teardown without the senders' unmap keys: %s", self.rank, e)
        finally:
            m.teardown_binding()
            self._mc = None

    def _collect_garbage(self) -> None:
        if self._garbage and self._janitor is not None:
            self._janitor.delete(self._garbage)
        self._garbage = []

    def _teardown(self) -> None:
        self._close_arm_socket()
        if self._watch is not None:
            self._watch.close()
            self._watch = None
        if self._janitor is not None:
            self._janitor.close()
            self._janitor = None
        for imp in self._pull_imports.values():
            try:
                imp.close()
            except Exception:
                pass
        self._pull_imports = {}
        try:
            self._leave_nvls()
        except Exception:
            logger.exception("receiver %d: multicast teardown", self.rank)
        srv = self._fd_server
        if srv is not None:
            srv.close()
            self._fd_server = None
        if self._board is not None:
            self._board.close()
            self._board = None
        self.session = None
        self._pg = None
        self._garbage = []

