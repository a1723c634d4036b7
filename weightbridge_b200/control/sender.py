"""Trainer-side sender: ``WeightSender(transfer_mode, receiver_urls).connect(meta); .send(sd)``.

connect (once, or to reshard):
  1. all-gather every sender's metadata over the trainer group;
  2. sender rank 0 queries ``/wbridge/metadata`` of every rollout URL, hosts the session
     store (OS-chosen port), computes the load-balanced source assignment and the plan
     digest of every (sender, receiver) pair, and POSTs ``/wbridge/connect``;
  3. every sender joins the store, reads the receivers' exported memory tables, opens
     the CUDA IPC handles of the receivers it writes to and a liveness connection to each;
     rank 0 connects its arm channel to every worker.
send (each sync):
  1. rank 0 arms the workers: one ZMQ message each (``arm="direct"``) or a POST of
     ``/wbridge/receive`` per rollout server (``arm="http"``); the schedulers call
     ``request_update`` when they can take new weights;
  2. the first send binds the state_dict, compiles the plan against the receivers'
     addresses and uploads the work tables; later sends reuse them;
  3. wait for every target's ``ready`` key; senders sharing split fp8 blocks exchange the
     blocks' amax; launch ONE transfer kernel (peer stores + fused layout transform / fp8
     quantisation + epoch flags), wait for it, publish ``done`` with the kernel's status.
     The wire modes pack and send chunk by chunk instead (``control/wires.py``).

Parity: ``wbridge/frontend/sender.py:7-26`` and ``wbridge/backend/direct_sender.py:16-211``
(``transfer_mode`` ``gpu_direct`` / ``cpu_direct``, rank-0 HTTP control, dedup).  The
payload path is new: no pack buffer, no NCCL ``isend``; ``cpu_direct`` works (the
reference's ``CPUDirectSender.send`` is a stub).
"""
from __future__ import annotations

import logging
import os
import socket
import threading
import time
import uuid
from dataclasses import dataclass, field
from datetime import timedelta
from typing import Any, Iterable

import numpy as np
import torch
import torch.distributed as dist

from ..core.binding import bind
from ..core.plan import (PhysBinding, PlanBoundsError, Tables, lower_ops, multicast_ok, phys_binding, plan_digest,
                         plan_pair, storage_ranges, validate_tables)
from ..core.plancache import PlanCache, plan_key, relative_binding
from ..core.shard import WeightData, covered_numel, shard_numel
from ..utils.config import WIRE_MODES, TransferConfig, normalize_mode
from .assign import assign_sources, restrict
from ..utils.trace import nvtx_range
from .protocol import PROTOCOL_VERSION, gpu_id
from .session import Janitor, PeerError, Session, SessionTimeout, local_address
from .board import digest_word

logger = logging.getLogger(__name__)


class TransferError(RuntimeError):
    pass


@dataclass
class SyncStats:
    epoch: int
    device_ms: float = 0.0          # transfer kernel, CUDA events on the transfer stream
    host_ms: float = 0.0            # whole send() call
    wait_ready_ms: float = 0.0
    exchange_ms: float = 0.0        # split fp8 blocks: amax pass and the exchange between senders
    bytes_read: int = 0
    bytes_written: int = 0
    receivers: list[int] = field(default_factory=list)
    status: int = 0
    link_gbs: float = 788.0         # bandwidth the fraction below is taken against (measured peer peak)
    marks: dict = field(default_factory=dict)   # time.perf_counter() at the sync's steps (start, done, armed, end)

    @property
    def gbs(self) -> float:
        """Bytes written per second of device time (GB/s)."""
        return self.bytes_written / (self.device_ms * 1e6) if self.device_ms > 0 else 0.0

    @property
    def link_fraction(self) -> float:
        """Achieved share of the per-GPU link bandwidth ``link_gbs``."""
        return self.gbs / self.link_gbs if self.link_gbs else 0.0

    def to_dict(self) -> dict:
        d = dict(self.__dict__)
        d["gbs"], d["link_fraction"] = round(self.gbs, 2), round(self.link_fraction, 4)
        return d


_HTTP = None


def _http():
    """A shared ``requests.Session``: keep-alive connections to the rollout servers, so the
    per-sync ``/wbridge/receive`` arm does not pay a TCP handshake."""
    global _HTTP
    if _HTTP is None:
        import requests
        _HTTP = requests.Session()
        _HTTP.ConnectionError = requests.ConnectionError
    return _HTTP


def _get_with_retry(http, url: str, timeout_s: float):
    """GET with bounded retries while the rollout server is still starting up."""
    deadline = time.monotonic() + timeout_s
    delay = 0.05
    while True:
        try:
            resp = http.get(url, timeout=timeout_s)
            resp.raise_for_status()
            return resp
        except http.ConnectionError:
            if time.monotonic() + delay > deadline:
                raise
            time.sleep(delay)
            delay = min(delay * 2, 1.0)


class WeightSender:
    """One trainer rank's side of the weight sync.

    ``transfer_mode``: ``gpu_direct`` (aliases ``p2p``, ``ipc``), ``nvls``, ``nccl`` or
    ``cpu_direct`` (``cpu``, ``gloo``).  ``receiver_urls``: the rollout servers hosting a
    ``WeightReceiverController``.  ``group``: the trainer process group whose ranks all send
    (default: the default group, or a single sender without torch.distributed).  ``config``:
    a ``TransferConfig`` (default: from ``WBRIDGE_*`` environment variables).

    Every rank calls ``connect(metadata)`` once and ``send(state_dict)`` after each update;
    ``metadata`` describes the rank's shards as logical HF boxes and ``state_dict`` holds
    tensors or views of them (``MegatronLayout.to_wb`` / ``FSDPLayout.to_wb`` give both).
    """

    def __init__(self, transfer_mode: str, receiver_urls: list[str], group: Any = None,
                 config: TransferConfig | None = None):
        self.transfer_mode = transfer_mode
        self.config = config or TransferConfig.from_env(mode=transfer_mode)
        self.config.mode = normalize_mode(transfer_mode)
        self.receiver_urls = list(receiver_urls)
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world_size = dist.get_world_size(group)
        else:
            self.rank, self.world_size = 0, 1
        self.connected = False
        self.metadata: WeightData | None = None
        self.session: Session | None = None
        self.epoch = 0
        self.targets: dict[int, list[str]] = {}
        self.overlaps: dict[int, WeightData] = {}
        self.history: list[SyncStats] = []
        self._program = None
        self._program_key = None
        self._routes: list[tuple[list[int], int]] = []   # (receivers one store reaches, bytes) of the program
        self._progs: dict[tuple, tuple] = {}        # compiled programs by (bound tensors, entry subset)
        self._imports: dict[int, Any] = {}
        self._rinfo: dict[int, dict] = {}
        self._ops_cache: dict[tuple, list] = {}     # plan ops per (receiver, bindings, names)
        self._plan_cache = PlanCache(self.config.plan_cache_dir) if self.config.plan_cache_dir else None
        self._bind_version = 0                       # bumped whenever the bound tensors change
        self._published_key = None                   # pull: the tensors whose memory was last exported
        self.uncovered: dict[int, list[str]] = {}    # rank 0, after connect: worker -> entries no sender fills
        self._xchg = None                            # split fp8 blocks shared with other senders
        self._writes_nothing = False                 # pull direction: senders store nothing
        self._overlap_nbytes: dict = {}              # bytes per entry subset (pull stats), per session
        self._board = None                           # same-host handshake words (control/board.py)
        self.direction = "push"                      # resolved at connect (session_direction)
        self._piece_pos = np.zeros(0, dtype=np.int64)
        self._arm_sock = None                        # rank 0, arm="direct": ROUTER to every receiver worker
        self._arm_idents: dict[int, bytes] = {}
        self._arm_error: str | None = None
        self._watch = None                           # liveness connections to the workers
        self._side = None                            # janitor: deletes and error writes off the critical path
        self._mc: dict = {}                          # nvls: multicast objects by replica group
        self._mc_created: list = []
        self._stream = self._ev = None               # transfer stream and its timing events (device tensors)
        self._pool = None                            # send_async's single worker thread
        self._snap = self._snap_key = self._snap_future = None   # send_async(snapshot=True) buffers
        self._wire_sets: dict = {}                   # wire modes: compiled wire sets by entry subset
        self._subsets_published: set[str] = set()   # wire modes, rank 0: subset digests in the session

    # -- collectives on the trainer group (no-ops for a single sender) -------------------
    def _all_gather(self, obj):
        if self.world_size == 1:
            return [obj]
        out = [None] * self.world_size
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def _broadcast(self, obj):
        if self.world_size == 1:
            return obj
        lst = [obj]
        src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
        dist.broadcast_object_list(lst, src=src, group=self.group)
        return lst[0]

    # -- connect ---------------------------------------------------------------------------
    def connect(self, sender_metadata: WeightData) -> None:
        if self.connected:
            self.disconnect()
        if self._board is not None:
            self._board.close()
            self._board = None
        self.metadata = sender_metadata
        self._rinfo = {}
        cfg = self.config
        metas = self._all_gather(sender_metadata.to_jsonable())
        self._sender_devices = self._all_gather(torch.cuda.current_device() if torch.cuda.is_available() else -1)
        self._sender_hosts = self._all_gather(socket.gethostname())
        self._sender_gpus = self._all_gather(gpu_id(torch.cuda.current_device()) if torch.cuda.is_available() else None)
        info = None
        if self.rank == 0:
            try:
                info = self._connect_rank0(metas)
            except Exception as e:   # every rank fails together instead of waiting in the broadcast
                info = {"error": f"rank 0 could not set up the session: {type(e).__name__}: {e}"}
        info = self._broadcast(info)
        if info.get("error"):
            raise TransferError(info["error"])
        cfg.mode = info["mode"]                      # resolved by rank 0 when it was "auto"
        addr, port, world = info["address"], info["port"], info["world_size"]
        if self.rank != 0:
            self.session = Session(addr, port, is_master=False, timeout_s=cfg.connect_timeout_s)
        self.world_total = world
        sess = self.session
        if self.rank != 0:
            from .board import SyncBoard
            self._board = SyncBoard.attach(sess.get_json("board", cfg.connect_timeout_s))
        assignment = sess.get_json("assign")
        mine = assignment.get(str(self.rank), {})
        self.targets = {int(r): names for r, names in mine.items() if names}
        rmetas = {int(k): WeightData(v) for k, v in info["receivers"].items()}
        self._all_receivers = set(rmetas)
        self.overlaps = {r: WeightData.compute_overlap(restrict(sender_metadata, names), rmetas[r])
                         for r, names in self.targets.items()}
        self._overlap_nbytes = {}
        self._xchg = self._exchange_plan(metas, assignment, rmetas)
        self.direction = session_direction(cfg, rmetas.values())
        # pulling, this sender never writes into its workers' memory, so a sync need not wait
        # for them to be idle (each loads when it is)
        self._writes_nothing = self.direction == "pull"
        # receivers publish their memory tables once they joined the store
        for r in self.targets:
            try:
                self._rinfo[r] = sess.get_json(f"recv/{r}", cfg.connect_timeout_s)
            except (SessionTimeout, PeerError) as e:
                raise TransferError(str(e)) from None
        if any(i.get("late") for i in self._rinfo.values()):
            self._writes_nothing = False           # late binders publish their memory with ready
        if cfg.mode == "nvls":
            try:
                self._setup_multicast(sess, info, assignment)
            except BaseException:
                self._teardown_multicast()       # nothing of this process stays bound to an object
                raise
        if cfg.mode in WIRE_MODES:
            # the group needs every rank: join it only once every receiver verified the plan
            everyone = sorted(rmetas)
            try:
                sess.wait_checked([f"verified/{r}" for r in everyone], cfg.connect_timeout_s,
                                  "receivers to verify the plan")
            except (SessionTimeout, PeerError) as e:
                raise TransferError(str(e)) from None
            self._pg = wire_group(cfg.mode, sess, self.rank, world, cfg.connect_timeout_s, addr)
        else:
            self._open_receivers()
        try:
            sess.wait_checked([f"joined/{r}" for r in self.targets], cfg.connect_timeout_s, "receivers to join")
        except (SessionTimeout, PeerError) as e:
            raise TransferError(str(e)) from None
        self._open_watch(addr, port)
        self.epoch = 0
        self._program = None
        self._program_key = None
        self._progs = {}
        self._published_key = None                   # the new session has no exported memory yet
        self._wire_sets = {}
        self._subsets_published = set()              # a new session holds none of them
        self.connected = True
        logger.info("sender %d connected: %d receiver targets, mode=%s", self.rank, len(self.targets), cfg.mode)

    def _open_watch(self, addr: str, port: int) -> None:
        """Liveness connections to every target worker (``control/liveness.py``) and a side
        channel to publish a lost worker's error while this thread waits on the session."""
        from .liveness import PeerWatch
        self._side = Janitor(addr, port, self.config.connect_timeout_s)
        self._watch = PeerWatch(self._receiver_lost)
        for r in sorted(self.targets):
            host, lport = self._rinfo[r]["live"]
            try:
                self._watch.add(PeerWatch.connect(host, int(lport), self.rank, self.config.connect_timeout_s), r)
            except OSError as e:
                raise TransferError(f"cannot reach receiver {r}'s liveness port {host}:{lport}: {e}") from None

    def _receiver_lost(self, r: int) -> None:
        """A target worker's process is gone: fail the waits for its keys now."""
        e = self.epoch + 1
        self._side.set_error([f"ready/{r}/{e}", f"pulled/{r}/{e}"],
                             f"receiver {r} left the session (its connection to sender {self.rank} closed)")

    def _close_watch(self) -> None:
        if self._watch is not None:
            self._watch.close()
            self._watch = None
        if self._side is not None:
            self._side.close()
            self._side = None

    def _exchange_plan(self, metas: list[dict], assignment: dict, rmetas: dict[int, WeightData]):
        """The split fp8 blocks this sender shares with other senders (``core/splitq.py``),
        or ``None``: nothing to exchange before a launch."""
        from ..core.splitq import exchange_plan
        if not any(any((m.quant(n) or {}).get("format") == "fp8_block" for n in m.names()) for m in rmetas.values()):
            return None
        plan = {int(s): {int(r): n for r, n in rs.items()} for s, rs in assignment.items()}
        x = exchange_plan(self.rank, [WeightData(m) for m in metas], plan, rmetas)
        return x if x is not None and x.keys else None

    def _split_amax(self, epoch: int, partial: np.ndarray) -> np.ndarray:
        """Split blocks: publish this sender's per-block amax, merge the co-owners' and return
        the block amax of every piece.  Raises ``SessionTimeout`` / ``PeerError``."""
        x, sess = self._xchg, self.session
        vals = x.local(partial, self._piece_pos)
        sess.set(f"amax/{self.rank}/{epoch}", vals.tobytes())
        if x.co_owners:
            blobs = sess.wait_checked([f"amax/{s}/{epoch}" for s in x.co_owners], self.config.sync_timeout_s,
                                      f"senders {x.co_owners} to share the amax of split fp8 blocks")
            vals = x.merge(vals, {s: np.frombuffer(b, dtype=np.float32) for s, b in zip(x.co_owners, blobs)})
        if epoch > 1:        # every co-owner published this epoch's key, so read the previous one
            sess.delete(f"amax/{self.rank}/{epoch - 1}")
        return vals[self._piece_pos]

    def _connect_rank0(self, metas: list[dict]) -> dict:
        cfg = self.config
        http = _http()
        receivers: dict[int, dict] = {}
        counts = []
        base = self.world_size
        where = []                                   # (host, device) of every worker
        rgpus: dict[int, str | None] = {}
        for url in self.receiver_urls:
            resp = _get_with_retry(http, f"{url}/wbridge/metadata", cfg.http_timeout_s)
            workers = sorted(resp.json(), key=lambda w: w["rank"])
            for i, w in enumerate(workers):
                receivers[base + i] = w["metadata"]
                where.append((w.get("host"), str(w.get("device", ""))))
                rgpus[base + i] = w.get("gpu")
            counts.append(len(workers))
            base += len(workers)
        if cfg.mode == "auto":
            cfg.mode = self._auto_mode(where)
        world = self.world_size + sum(counts)
        addr = cfg.master_address
        if addr in ("", "auto"):
            from urllib.parse import urlparse
            hosts = {urlparse(u).hostname for u in self.receiver_urls}
            addr = "127.0.0.1" if hosts <= {"127.0.0.1", "localhost", "::1"} else local_address()
        self.session = Session(addr, cfg.master_port, is_master=True, timeout_s=cfg.connect_timeout_s)
        sess = self.session
        smeta_objs = [WeightData(m) for m in metas]
        rmeta_objs = {r: WeightData(m) for r, m in receivers.items()}
        # multicast: every replica of a layout takes each entry from the same sender; otherwise a
        # replicated entry comes from a trainer rank on the worker's own GPU where there is one
        plan = assign_sources(smeta_objs, rmeta_objs, cfg.load_balance, replica_consistent=cfg.mode == "nvls",
                              sender_gpus=self._sender_gpus, receiver_gpus=rgpus)
        sess.set_json("senders/meta", metas)
        sess.set("direction", session_direction(cfg, rmeta_objs.values()))
        sess.set("wire_chunk", str(int(cfg.wire_chunk_bytes)))      # receivers cut their wires alike
        sess.set_json("assign", {str(s): {str(r): n for r, n in rs.items()} for s, rs in plan.items()})
        covered: dict[tuple[int, str], int] = {}
        for s, rs in plan.items():
            for r, names in rs.items():
                ov = WeightData.compute_overlap(restrict(smeta_objs[s], names), rmeta_objs[r])
                sess.set(f"digest/{s}/{r}", plan_digest(ov))
                rm = rmeta_objs[r]
                for n, regions, _dt in ov:
                    if (rm.quant(n) or {}).get("role") == "scale":
                        continue
                    k = sum(covered_numel(reg, rm.shards(n)) for reg in regions)
                    covered[(r, n)] = covered.get((r, n), 0) + k
        self.uncovered = _uncovered(rmeta_objs, covered)
        if self.uncovered:
            msg = ", ".join(f"worker {r}: {len(v)} entries (e.g. {v[0]})" for r, v in sorted(self.uncovered.items()))
            if cfg.require_full_coverage:
                raise TransferError(f"no sender holds some of the rollout's weights: {msg}")
            logger.warning("no sender holds some of the rollout's weights (they keep their values): %s", msg)
        session_id = uuid.uuid4().hex
        # peers on one host: per-sync handshake words in shared memory (control/board.py)
        me = socket.gethostname()
        if cfg.mode in ("gpu_direct", "nvls") and all(h == me for h in self._sender_hosts) \
                and all(h == me for h, _d in where):
            from .board import SyncBoard
            self._board = SyncBoard.create(session_id, self.world_size, sum(counts))
        sess.set_json("board", self._board.describe() if self._board is not None else {})
        backend = cfg.mode
        base = self.world_size
        for url, count in zip(self.receiver_urls, counts):
            resp = http.post(f"{url}/wbridge/connect", timeout=cfg.http_timeout_s, json={
                "master_address": addr, "master_port": sess.port, "base_rank": base, "world_size": world,
                "group_name": "wbridge", "sender_world_size": self.world_size, "backend": backend,
                "session": session_id, "protocol": PROTOCOL_VERSION})
            resp.raise_for_status()
            if resp.json().get("status") != "success":
                return {"error": f"receiver {url} refused connect: {resp.json()}"}
            base += count
        if cfg.arm == "direct":
            self._open_arm_channel(sorted(receivers))
        return {"address": addr, "port": sess.port, "world_size": world, "mode": cfg.mode,
                "receivers": {str(r): m for r, m in receivers.items()}, "session": session_id}

    def _auto_mode(self, where: list[tuple[str | None, str]]) -> str:
        """``transfer_mode="auto"``: ``gpu_direct`` when every sender and worker holds CUDA
        tensors on one host, ``nccl`` when they are on GPUs of several hosts, else
        ``cpu_direct``."""
        gpus = all(d >= 0 for d in self._sender_devices) and all(dev.startswith("cuda") for _h, dev in where)
        hosts = set(self._sender_hosts) | {h for h, _d in where}
        mode = ("gpu_direct" if len(hosts) == 1 else "nccl") if gpus else "cpu_direct"
        logger.info("transfer_mode auto -> %s (hosts %s)", mode, sorted(h for h in hosts if h))
        return mode

    def _open_arm_channel(self, receivers: list[int]) -> None:
        """``arm="direct"``: connect one ROUTER to every receiver worker's arm socket (their
        endpoints are in the session) and wait until each connection is up, so that a later
        arm either reaches the worker or fails at once (``ROUTER_MANDATORY``: a worker whose
        process is gone is unroutable) instead of queueing."""
        import zmq
        cfg = self.config
        self._close_arm_channel()
        sock = zmq.Context.instance().socket(zmq.ROUTER)
        sock.setsockopt(zmq.LINGER, 0)
        sock.setsockopt(zmq.ROUTER_MANDATORY, 1)
        sock.setsockopt(zmq.IMMEDIATE, 1)          # a route exists only while its connection is up
        try:
            idents = {}
            for r in receivers:
                info = self.session.get_json(f"recv/{r}", cfg.connect_timeout_s)
                sock.connect(info["arm"])
                idents[r] = f"wbarm-{r}".encode()
            pending, deadline = set(receivers), time.monotonic() + cfg.connect_timeout_s
            while pending:
                for r in sorted(pending):
                    try:
                        sock.send_multipart([idents[r], b"{}"], zmq.NOBLOCK)     # probe, ignored by the worker
                        pending.discard(r)
                    except zmq.ZMQError:
                        pass
                if pending and time.monotonic() > deadline:
                    raise TransferError(f"receivers {sorted(pending)} unreachable on their arm sockets")
                if pending:
                    time.sleep(0.002)
        except BaseException:
            sock.close(0)
            raise
        self._arm_sock, self._arm_idents = sock, idents

    def _close_arm_channel(self) -> None:
        sock, self._arm_sock, self._arm_idents = self._arm_sock, None, {}
        if sock is not None:
            sock.close(0)

    def _open_receivers(self) -> None:
        from ..parallel.ipc import ImportTable
        host, pid = socket.gethostname(), os.getpid()
        for r, info in self._rinfo.items():
            if info.get("mode") not in ("gpu_direct", "nvls"):
                raise TransferError(f"receiver {r} joined in mode {info.get('mode')}")
            if info.get("late"):
                continue            # bound at its first update; opened in _resolve_bindings
            if info["host"] != host:
                raise TransferError(f"receiver {r} is on host {info['host']}: gpu_direct needs one node")
            if info.get("device", 0) < 0 and info["pid"] != pid:
                raise TransferError(f"receiver {r} holds host memory in another process; use cpu_direct")
            self._imports[r] = ImportTable(info["allocs"], same_process=(info["pid"] == pid))

    # -- NVLink multicast (mode "nvls") --------------------------------------------------------
    def _setup_multicast(self, sess: Session, info: dict, assignment: dict) -> None:
        """Rank 0 finds replica groups and creates one multicast object per group; every
        sender of a group adds its device and backs the object with scratch (unless a replica on
        its GPU already does), then maps it."""
        from ..parallel.nvls import McMember, nvls_supported, replica_groups
        cfg = self.config
        self._mc: dict[int, tuple] = {}
        self._mc_created: list = []
        if self.rank == 0:
            everyone = sorted(int(r) for r in info["receivers"])
            try:
                allinfo = {r: sess.get_json(f"recv/{r}", cfg.connect_timeout_s) for r in everyone}
            except (SessionTimeout, PeerError) as e:
                raise TransferError(str(e)) from None
            plan = {int(s): {int(r): n for r, n in rs.items()} for s, rs in assignment.items()}
            groups = []
            dev0 = torch.cuda.current_device()
            for gid, reps in enumerate(replica_groups(allinfo)):
                senders = [s for s, rs in plan.items()
                           if all(r in rs for r in reps) and all(rs[r] == rs[reps[0]] for r in reps)]
                # a sender on a replica's GPU shares that device's membership (the replica's pool
                # backs it); every other member needs a GPU of its own
                rep_devs = [allinfo[r]["device"] for r in reps]
                colocated = [s for s in senders if self._sender_devices[s] in rep_devs]
                extra = [self._sender_devices[s] for s in senders if s not in colocated]
                distinct = len(set(rep_devs)) == len(rep_devs) and len(set(extra)) == len(extra)
                if not senders or not nvls_supported(dev0) or not distinct:
                    logger.warning("replica group %s goes unicast: %s", reps,
                                   "no sender writes the same entries to all of it" if not senders else
                                   "two replicas, or two senders off the replicas, share a GPU" if not distinct
                                   else "the GPU reports no NVLink multicast")
                    continue
                size = int(allinfo[reps[0]]["pool"]["size"])
                m = McMember(gid, size, dev0)
                m.create(num_devices=len(rep_devs) + len(extra))
                self._mc_created.append(m)
                groups.append({"id": gid, "replicas": reps, "senders": senders, "colocated": colocated,
                               "size": size, "addr": m.server.address})
            sess.set_json("nvls/plan", {"groups": groups})
        plan = sess.get_json("nvls/plan", cfg.connect_timeout_s)
        dev = torch.cuda.current_device()
        for g in plan["groups"]:
            if self.rank not in g["senders"]:
                continue
            creator = next((m for m in self._mc_created if m.group == g["id"]), None)
            m = creator if creator is not None else McMember(g["id"], g["size"], dev)
            self._mc[g["id"]] = (m, g)           # tracked from here on: teardown undoes every stage
            if creator is None:
                m.join(g["addr"])
            shared = self.rank in g.get("colocated", [])      # a replica on this GPU backs the object
            if not shared:
                m.add_device()
            sess.set(f"nvls/{g['id']}/added/{self.rank}", "1")
            members = g["replicas"] + g["senders"]
            sess.wait_checked([f"nvls/{g['id']}/added/{x}" for x in members], cfg.connect_timeout_s,
                              "multicast members to add their devices")
            if not shared:
                m.bind_scratch()
            sess.set(f"nvls/{g['id']}/bound/{self.rank}", "1")
            sess.wait_checked([f"nvls/{g['id']}/bound/{x}" for x in members], cfg.connect_timeout_s,
                              "multicast members to bind memory")
            m.map()
        logger.info("sender %d: %d multicast group(s)", self.rank, len(self._mc))

    def _leave_session(self) -> None:
        """The session store lives in rank 0's process: rank 0 keeps it up until every other
        sender rank has left (bounded by the sync deadline), so a rank still finishing its last
        sync, reading its workers' keys, is not cut off by rank 0 leaving first.  The other
        ranks say they left."""
        sess = self.session
        if sess is None or self.world_size <= 1:
            return
        try:
            if self.rank == 0:
                sess.wait([f"left/{r}" for r in range(1, self.world_size)], self.config.sync_timeout_s,
                          "the other sender ranks to leave")
            else:
                sess.set(f"left/{self.rank}", "1")
        except Exception as e:       # a rank that never leaves (gone) costs the wait, nothing else
            logger.warning("sender %d: leaving the session: %s", self.rank, e)

    def _teardown_multicast(self) -> None:
        """Unmap, tell the group, and unbind only once every sender of the group unmapped
        (no multimem store can then reach this device's backing).  Also undoes a set-up that
        stopped half way: members that never mapped still report ``unmapped``."""
        mc = self._mc
        sess = self.session
        for m, g in mc.values():
            try:
                m.teardown_mapping()
            finally:
                if sess is not None:
                    try:
                        sess.set(f"nvls/{g['id']}/unmapped/{self.rank}", "1")
                    except Exception:
                        logger.exception("sender %d: could not report the multicast unmap", self.rank)
        for m, g in mc.values():
            try:
                if sess is not None:
                    sess.wait([f"nvls/{g['id']}/unmapped/{x}" for x in g["senders"]], self.config.connect_timeout_s)
            except Exception:
                logger.exception("sender %d: multicast group %d: waiting for the other senders to unmap",
                                 self.rank, g["id"])
            finally:
                m.teardown_binding()
        plan = {}
        if self._mc_created and sess is not None:
            try:
                plan = {g["id"]: g for g in sess.get_json("nvls/plan", 1.0)["groups"]}
            except Exception:
                logger.exception("sender %d: multicast plan unreadable at teardown", self.rank)
        for m in self._mc_created:
            if all(m is not x for x, _g in mc.values()):
                # created here, written by others: the store (held by this rank) stays up until
                # they unmapped, so the replicas can read the same keys before they unbind
                g = plan.get(m.group)
                try:
                    if g is not None:
                        sess.wait([f"nvls/{g['id']}/unmapped/{x}" for x in g["senders"]], self.config.connect_timeout_s)
                except Exception:
                    logger.exception("sender %d: multicast group %d: waiting for its senders to unmap", self.rank,
                                     m.group)
                finally:
                    m.teardown_binding()
        self._mc, self._mc_created = {}, []

    def _resolve_bindings(self, ready: dict[int, bytes]) -> bool:
        """Open the memory of workers that bound tensors after connect: late binders at their
        first update, and workers that called ``rebind`` (their ready key carries a new binding
        generation).  Both publish ``recvbind/<rank>`` before marking ready.  True if any
        changed (the compiled programs then refer to old memory)."""
        from ..parallel.ipc import ImportTable
        changed = False
        for r, info in self._rinfo.items():
            gen = int(ready[r]) if r in ready and ready[r].isdigit() else info.get("gen", 1)
            stale = info.get("late") and r not in self._imports
            if not stale and gen == info.get("gen", 1):
                continue
            try:
                info.update(self.session.get_json(f"recvbind/{r}", self.config.sync_timeout_s))
            except (SessionTimeout, PeerError) as e:
                raise TransferError(str(e)) from None
            old = self._imports.pop(r, None)
            if old is not None:
                old.close()
            self._imports[r] = ImportTable(info["allocs"], same_process=(info["pid"] == os.getpid()))
            changed = True
        return changed

    def reconnect(self) -> None:
        """Connect again with the last metadata, e.g. after a rollout worker restarted: a new
        session, fresh IPC mappings, epochs restarting at 1.  Plan ops are reused for every
        receiver whose physical binding did not change."""
        if self.metadata is None:
            raise RuntimeError("reconnect() needs a previous connect()")
        self.connect(self.metadata)

    def __enter__(self) -> "WeightSender":
        return self

    def __exit__(self, *exc) -> None:
        self.disconnect()

    def disconnect(self) -> None:
        """Leave the session (liveness connections say bye, IPC mappings close); waits for a
        sync started with ``send_async``."""
        pool = self._pool
        if pool is not None:
            pool.shutdown(wait=True)
            self._pool = None
        self._snap = self._snap_key = self._snap_future = None
        self._close_watch()
        self._close_arm_channel()
        self._teardown_multicast()
        self._leave_session()
        for imp in self._imports.values():
            imp.close()
        self._imports.clear()
        if self._board is not None:
            self._board.close()
            self._board = None
        self._program = None
        self.session = None
        self.connected = False

    # -- send ----------------------------------------------------------------------------------
    def _compile(self, state_dict, subset: frozenset | None = None) -> None:
        """Compile the push program for ``state_dict`` (entries restricted to ``subset``)."""
        cfg = self.config
        self._routes = []
        if not self.targets:
            self._program = None
            return
        binding = bind(self.metadata, state_dict)
        device = binding.device
        sphys, ptrs = relative_binding(binding)      # address-free: plans survive reallocation
        src_base = ptrs.__getitem__
        sjson = sphys.to_json()
        skey = _digest(sjson)
        pull = self.direction == "pull"
        if not pull:
            self._bind_version += 1
        elif self._published_key != self._key(state_dict):   # new tensors: export them again
            self._bind_version += 1
            self._publish_sender_memory(binding, device)
            self._published_key = self._key(state_dict)
        parts, flags, dst_ranges = [], [], []
        covered: set[int] = set()
        routes: list[tuple[list[int], int]] = []
        for m, g in self._mc.values():
            reps = g["replicas"]
            rep = reps[0]
            names = [n for n in self.targets[rep] if subset is None or n in subset]
            rphys = PhysBinding.from_json(self._rinfo[rep]["binding"])
            ops = plan_pair(sphys, rphys, names=names)
            mc_base = lambda a, va=m.va: va
            mc_ops = [o for o in ops if multicast_ok(o, src_base, mc_base)]
            uni_ops = [o for o in ops if not multicast_ok(o, src_base, mc_base)]
            mct = lower_ops(mc_ops, src_base, mc_base, item_bytes=cfg.item_bytes, multicast=True)
            parts.append(mct)
            routes.append((list(reps), mct.bytes_written))     # one multimem store reaches every replica
            dst_ranges.append((m.va, m.va + m.size))
            for r in reps:
                info, imp = self._rinfo[r], self._imports[r]
                if uni_ops:          # casts, quantised blocks, unaligned copies: one store per replica
                    parts.append(lower_ops(uni_ops, src_base, imp.base, item_bytes=cfg.item_bytes, receiver=r))
                    routes.append(([r], parts[-1].bytes_written))
                dst_ranges += [(imp.base(i), imp.base(i) + int(a["size"])) for i, a in enumerate(info["allocs"])]
            # the replicas' pools are laid out alike, flag words included: one multicast release
            # store (bit 0 marks the address as multicast) reaches every replica's word
            _falloc, foff, _w = self._rinfo[rep]["flags"]
            flags.append((m.va + foff + 8 * self.rank) | 1)
            covered |= set(reps)
        for r, names in sorted(self.targets.items()):
            if r in covered:
                continue
            if subset is not None:
                names = [n for n in names if n in subset]
            info = self._rinfo[r]
            imp = self._imports[r]
            ckey = (r, _digest(info["binding"]), skey, tuple(names))
            ops = self._ops_cache.get(ckey)
            rphys = PhysBinding.from_json(info["binding"])
            if ops is None and self._plan_cache is not None:
                dkey = plan_key(sjson, info["binding"], names)
                ops = self._plan_cache.get(dkey)
                if ops is None:
                    ops = plan_pair(sphys, rphys, names=names)
                    self._plan_cache.put(dkey, ops)
                self._ops_cache[ckey] = ops
            if ops is None:
                ops = plan_pair(sphys, rphys, names=names)
                self._ops_cache[ckey] = ops
            if pull:                       # receivers load the copies; quantised blocks stay pushed
                ops = [o for o in ops if o.kind in ("quant", "squant")]
            parts.append(lower_ops(ops, src_base, imp.base, item_bytes=cfg.item_bytes, receiver=r))
            routes.append(([r], parts[-1].bytes_written))
            falloc, foff, _w = info["flags"]
            flags.append(imp.base(falloc) + foff + 8 * self.rank)
            if info["allocs"]:
                dst_ranges += [(imp.base(i), imp.base(i) + int(a["size"])) for i, a in enumerate(info["allocs"])]
            else:                          # host memory of this process: the bound regions themselves
                dst_ranges += _phys_extents(rphys) + [(foff, foff + 8 * int(_w))]
        tables = _interleave(parts)
        self._routes = routes
        self._piece_pos = self._positions(tables)
        if cfg.validate_plan:
            validate_tables(tables, storage_ranges(state_dict.values()), dst_ranges)
            for f in flags:
                _check_flag(f, dst_ranges)
        from ..ops.executor import MODE_AUTO, MODE_VECTOR, HostProgram, LaunchConfig, TransferProgram
        if not len(tables):                # pull mode without quantised blocks: nothing to push
            self._program = None
            return
        if device.type == "cpu":
            if any(self._rinfo[r].get("device", 0) >= 0 for r in self.targets):
                raise TransferError("a CPU sender cannot store into GPU receivers; use cpu_direct")
            self._program = HostProgram(tables, flags)
            return
        lc = LaunchConfig(mode=cfg.kernel_mode, piece_bytes=cfg.piece_bytes, grid=cfg.grid or None)
        if (lc.mode == MODE_AUTO and len(tables.qwork)
                and any(int(self._rinfo[r].get("device", -1)) != device.index for r in self.targets)):
            # quant blocks stored into another GPU keep the register path (vector mode), the one
            # measured end to end at 0.863 of the peer peak (Qwen3-30B-A3B EP2 -> TP2).  One sender
            # into one peer, both quantisers run alike (0.878 / 0.881), but the sync with four
            # senders each storing into four peers (EP4 -> TP4) reached only 0.659 with the
            # tensor-map-fed one, a gap not yet profiled; it stays for blocks quantised locally
            lc.mode = MODE_VECTOR
        torch.cuda.set_device(device)
        self._program = TransferProgram(tables, device, flags, lc)
        self._stream = torch.cuda.Stream(device)
        self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    def _publish_sender_memory(self, binding, device) -> None:
        """Pull direction: export this sender's parameter memory for its receivers."""
        info = {"version": self._bind_version, "pid": os.getpid(), "host": socket.gethostname(),
                "device": device.index if device.type == "cuda" else -1}
        if device.type == "cuda":
            from ..parallel.ipc import ExportTable
            export = ExportTable(device)
            phys = phys_binding(binding, export.locate)        # locates (and exports) every allocation
            info.update({"allocs": export.to_json(), "binding": phys.to_json()})
            self._export = export
        else:                              # host memory: readable only inside this process
            info.update({"allocs": [], "binding": phys_binding(binding).to_json()})
        self.session.set_json(f"sendbind/{self.rank}", info)

    def _publish_subset(self, subset: frozenset | None) -> str:
        """Wire modes, rank 0: the digest the receivers look a partial sync's entries up by
        (``""``: every entry); each subset's names are written to the session once."""
        if subset is None:
            return ""
        names = sorted(subset)
        dg = _digest(names)[:16]
        if dg not in self._subsets_published:
            self.session.set_json(f"subset/{dg}", names)
            self._subsets_published.add(dg)
        return dg

    def _select_wire(self, state_dict, subset: frozenset | None) -> None:
        """Make the wire set of ``subset`` current (compiled on first use, on the full set's
        buffers); the last few subsets stay compiled."""
        ws = self._wire_sets.get(subset)
        if ws is None:
            if subset is not None and None not in self._wire_sets:
                self._select_wire(state_dict, None)           # its buffers serve every subset
            self._compile_wire(state_dict, subset)
            ws = self._wires
            if len(self._wire_sets) >= 8:
                self._wire_sets.pop(next(k for k in self._wire_sets if k is not None))
            self._wire_sets[subset] = ws
        self._wires = ws
        self._piece_pos = self._positions(ws.all_tables)

    def _compile_wire(self, state_dict, subset: frozenset | None = None) -> None:
        """Wire modes: every target's overlap (restricted to ``subset``) cut into chunks with
        two buffers per target (``control/wires.py``), packed by the C++ executor for host
        tensors and by one transfer-kernel launch per chunk for device tensors."""
        from ..core.wire import restrict_overlap
        from .wires import WireSet
        cfg = self.config
        binding = bind(self.metadata, state_dict)
        dev = binding.device
        if cfg.mode == "cpu_direct" and dev.type != "cpu":
            raise TransferError("cpu_direct sends host tensors; use nccl or gpu_direct for device tensors")
        if cfg.mode == "nccl" and dev.type != "cuda":
            raise TransferError("nccl mode sends device tensors; use cpu_direct for host tensors")
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
        overlaps, targets = self.overlaps, self.targets
        shared = None
        if subset is not None:
            overlaps = {r: restrict_overlap(ov, subset) for r, ov in overlaps.items()}
            targets = {r: [n for n in names if n in subset] for r, names in targets.items()}
            full = self._wire_sets.get(None)
            shared = full.buffers() if full is not None else None
        self._wires = WireSet.for_sender(phys_binding(binding), overlaps, targets, dev, cfg,
                                         storage_ranges(state_dict.values()), shared)
        self._piece_pos = self._positions(self._wires.all_tables)
        self._program = None
        if dev.type == "cuda" and self._stream is None:
            self._stream = torch.cuda.Stream(dev)
            self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    def _select(self, state_dict, subset: frozenset | None) -> None:
        """Make the program for (bound tensors, entry subset) current, compiling it on first
        use; the last few stay compiled, so alternating full and partial syncs do not
        recompile."""
        key = (self._key(state_dict), subset)
        if key == self._program_key:
            return
        if self.direction == "pull":            # the receivers pull from the last published memory:
            # programs of other tensors are dropped (a switch of tensors publishes again)
            self._progs = {k: v for k, v in self._progs.items() if k[0] == key[0]}
        hit = self._progs.pop(key, None)
        if hit is None:
            self._compile(state_dict, subset)
            hit = (self._program, self._piece_pos, self._routes)
        self._progs[key] = hit
        while len(self._progs) > 4:
            self._progs.pop(next(iter(self._progs)))
        self._program, self._piece_pos, self._routes = hit
        self._program_key = key

    def _positions(self, tables: Tables) -> np.ndarray:
        if not len(tables.pieces):
            return np.zeros(0, dtype=np.int64)
        if self._xchg is None:
            raise TransferError("the plan has split fp8 blocks but the exchange plan has none")
        return self._xchg.positions(tables.piece_keys)

    def _key(self, state_dict) -> bytes:
        """Identity of the bound tensors: per entry, in dict order, the name's hash and the data
        pointers of its tensor (lists of views included), so a rebound or reallocated tensor
        recompiles the plan.  One C++ pass over the dict (``state_key``)."""
        from ..ops._ext import ext
        if isinstance(state_dict, dict):
            return ext().state_key(state_dict)
        return ext().state_key(dict(state_dict))

    def launch(self, state_dict: dict[str, Any], stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue this sender's transfer kernel on ``stream`` with no HTTP arm, no handshake
        and no host synchronisation.  For callers that already know the rollout side is
        idle (and for device-timed benchmarks): the receivers' epoch flags are not touched,
        so a later ``send`` still pairs with ``request_update``.  Blocks split across senders
        are quantised with the block amax exchanged by the last ``send``, and the receivers'
        memory is the one known at the last ``send`` (after a worker's ``rebind``, run a
        ``send`` first)."""
        if not self.connected:
            raise RuntimeError("WeightSender.launch requires connect() first")
        if self.config.mode in WIRE_MODES:
            raise RuntimeError("launch() stores into receiver memory; wire modes use send()")
        if any(info.get("late") and r not in self._imports for r, info in self._rinfo.items()):
            raise RuntimeError("launch() needs every receiver's memory; run one send() first")
        self._select(state_dict, None)
        if self._program is not None and len(self._program.tables):
            if self._program.device.type == "cpu":
                self._program.launch(0, signal=False)
            else:
                self._program.launch(0, stream or torch.cuda.current_stream(self._program.device), signal=False)

    @property
    def program(self):
        """The compiled transfer program (tables, grid, byte counts), once compiled."""
        return self._program

    @property
    def delivered_bytes(self) -> int:
        """Bytes the compiled push program lands in receivers per sync: a multicast store
        counts once per replica it reaches."""
        return sum(n * len(rs) for rs, n in self._routes) if self._program is not None else 0

    def routes(self) -> list[dict]:
        """Where the compiled push program's bytes go: one record per receiver (unicast) or per
        replica group (multicast), with the GPU ordinals on both ends."""
        if self._program is None:
            return []
        src = self._program.device.index if self._program.device.type == "cuda" else -1
        return [{"src": src, "dst": [int(self._rinfo[r].get("device", -1)) for r in rs], "bytes": int(n),
                 "multicast": len(rs) > 1} for rs, n in self._routes if n]

    def _arm(self, epoch: int) -> threading.Thread | None:
        """Arm sync ``epoch`` on every receiver worker (rank 0 only).  A failed arm is written
        into every receiver's ready key, so all senders stop waiting at once.

        ``arm="direct"``: one ZMQ message per worker on the connections opened at connect; a
        worker that cannot take the sync writes why into its own ready key.
        ``arm="http"`` (the reference's protocol): POST ``/wbridge/receive`` to every rollout
        server from a helper thread.  Only the request reaching the workers is on the critical
        path (they then report ready through the session); the responses are checked after
        the ready wait."""
        self._arm_error = None
        receivers = sorted(self._all_receivers)
        if self._arm_sock is not None:
            import zmq
            payload = f'{{"epoch":{epoch}}}'.encode()
            for r, ident in self._arm_idents.items():
                try:
                    self._arm_sock.send_multipart([ident, payload], zmq.NOBLOCK)
                except zmq.ZMQError as e:
                    self._arm_error = f"arming the rollout side failed: receiver {r} unreachable ({e})"
                    self.session.set_error([f"{k}/{x}/{epoch}" for x in receivers for k in ("ready", "pulled")],
                                           self._arm_error)
                    break
            return None
        urls, timeout = list(self.receiver_urls), self.config.http_timeout_s

        def run():
            try:
                http = _http()
                with nvtx_range("wbridge.send/arm"):
                    for url in urls:
                        resp = http.post(f"{url}/wbridge/receive", timeout=timeout)
                        resp.raise_for_status()
                        if resp.json().get("status") != "success":
                            raise TransferError(f"receiver {url} refused the sync: {resp.json()}")
            except Exception as e:
                self._arm_error = f"arming the rollout side failed: {type(e).__name__}: {e}"
                self.session.set_error([f"{k}/{r}/{epoch}" for r in receivers for k in ("ready", "pulled")],
                                       self._arm_error)

        th = threading.Thread(target=run, name="wbridge-arm", daemon=True)
        th.start()
        return th

    def _fail_epoch(self, epoch: int, message: str) -> None:
        """Tell this epoch's receivers (and the senders sharing split fp8 blocks with this
        one) that no data is coming: they stop waiting at once."""
        if self.session is not None:
            keys = [f"done/{self.rank}/{r}/{epoch}" for r in self.targets]
            if self._xchg is not None:
                keys.append(f"amax/{self.rank}/{epoch}")
            self.session.set_error(keys, f"sender {self.rank}: {message}")

    def send(self, state_dict: dict[str, Any], version: int | None = None,
             names: Iterable[str] | None = None) -> SyncStats:
        """One full sync: arm the rollout side, wait until every target receiver is ready,
        launch the transfer kernel, wait for it and report completion.  ``version`` (e.g. the
        training step) tags the weights: workers report it as ``weights_version``.  ``names``
        restricts the sync to those HF entries (e.g. skip frozen layers); every sender rank
        must pass the same set (push direction of ``gpu_direct`` and ``nvls`` only).  NVTX
        ranges mark the phases (``wbridge.send/arm``, ``/ready``, ``/transfer``)."""
        if self._pool is not None:     # after send_async: keep the call order
            return self.send_async(state_dict, version, names).result()
        subset = self._subset(names)
        with nvtx_range("wbridge.send"):
            return self._send(state_dict, -1 if version is None else int(version), subset)

    def send_async(self, state_dict: dict[str, Any], version: int | None = None,
                   names: Iterable[str] | None = None, snapshot: bool = False):
        """Start a sync and return at once with a ``concurrent.futures.Future`` of its
        ``SyncStats``: the handshake and the transfer run on a helper thread while the caller
        goes on (the next forward and backward only read the parameters).  The parameters
        must stay unchanged until ``future.result()`` returns - call it before the next
        optimizer step.  Syncs of one sender run one at a time, in call order.  The transfer
        is ordered after the work enqueued on the caller's current stream before this call.

        ``snapshot=True`` first copies the tensors (on the caller's current stream, into
        buffers this sender keeps: the memory of its shard once more) and syncs the copy, so
        the caller may update its parameters at once.  The copy waits for the previous
        snapshot sync to be done with the buffers."""
        subset = self._subset(names)
        if snapshot:
            prev = self._snap_future
            if prev is not None:
                prev.exception()              # wait; its error is its own future's
            state_dict = self._take_snapshot(state_dict)
        after = device = None
        if torch.cuda.is_available():
            device = torch.cuda.current_device()
            after = torch.cuda.Event()
            after.record(torch.cuda.current_stream(device))
        if self._pool is None:
            from concurrent.futures import ThreadPoolExecutor
            self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="wbridge-send")
        tag = -1 if version is None else int(version)

        def run():
            if device is not None:
                torch.cuda.set_device(device)         # the helper thread starts on device 0
            with nvtx_range("wbridge.send"):
                return self._send(state_dict, tag, subset, after)

        fut = self._pool.submit(run)
        if snapshot:
            self._snap_future = fut
        return fut

    def _take_snapshot(self, state_dict: dict[str, Any]) -> dict[str, Any]:
        """Copy ``state_dict``'s tensors (lists of views included) into this sender's snapshot
        buffers, allocated on first use and again when the tensors change."""
        key = self._key(state_dict)
        if self._snap_key != key:
            self._snap = {n: [torch.empty_like(t) for t in v] if isinstance(v, (list, tuple)) else torch.empty_like(v)
                          for n, v in state_dict.items()}
            self._snap_key = key
        src, dst = [], []
        for n, v in state_dict.items():
            if isinstance(v, (list, tuple)):
                src += list(v)
                dst += self._snap[n]
            else:
                src.append(v)
                dst.append(self._snap[n])
        torch._foreach_copy_(dst, src)
        return self._snap

    @staticmethod
    def _wait_after(stream, after, device) -> None:
        """Order ``stream`` after ``after`` (an event recorded by the caller, or a stream;
        ``None``: this thread's current stream on ``device``)."""
        if isinstance(after, torch.cuda.Event):
            stream.wait_event(after)
        else:
            stream.wait_stream(after if after is not None else torch.cuda.current_stream(device))

    def summary(self, last: int = 100) -> dict:
        """Median and 90th percentile of the last ``last`` syncs' host time, device time, wait
        for the workers and GB/s (``SyncStats``), for periodic logging."""
        hist = self.history[-last:]
        out: dict = {"syncs": len(hist)}
        if not hist:
            return out
        for f in ("host_ms", "device_ms", "wait_ready_ms", "exchange_ms", "gbs"):
            v = np.sort(np.array([getattr(h, f) for h in hist], dtype=np.float64))
            out[f] = {"p50": round(float(np.percentile(v, 50)), 3), "p90": round(float(np.percentile(v, 90)), 3)}
        out["bytes_written"] = hist[-1].bytes_written
        return out

    def _overlap_bytes(self, subset: frozenset | None) -> int:
        """Bytes of this sender's entries its targets receive (restricted to ``subset``),
        computed once per subset and session."""
        n = self._overlap_nbytes.get(subset)
        if n is None:
            n = sum(end - start for ov in self.overlaps.values() for start, end, name, _sh, _dt in ov.iter_with_intv()
                    if subset is None or name in subset)
            self._overlap_nbytes[subset] = n
        return n

    def _subset(self, names) -> frozenset | None:
        return None if names is None else frozenset(names)

    def _send(self, state_dict: dict[str, Any], version: int = -1, subset: frozenset | None = None,
              after: Any = None) -> SyncStats:
        """One sync: handshake, program selection, split-block exchange, transfer, completion.
        ``after``: the event or stream whose work the transfer must follow (default: this
        thread's current stream on the transfer's device)."""
        if not self.connected or self.metadata is None:
            raise RuntimeError("WeightSender.send requires connect() first")
        t0 = time.perf_counter()
        epoch = self.epoch + 1
        st = SyncStats(epoch=epoch, receivers=sorted(self.targets), link_gbs=self.config.link_gbs)
        st.marks["start"] = t0
        if self._writes_nothing:          # pulling: done is published before the arm (_transfer_direct)
            ready = []
        else:
            ready = self._handshake(epoch, version, subset, st)
        self._prepare(state_dict, subset, ready, epoch)
        st.marks["prepared"] = time.perf_counter()
        if len(self._piece_pos):          # split fp8 blocks: amax of every piece, then the exchange
            self._exchange_split_amax(epoch, st, after)
        if self.config.mode in WIRE_MODES:
            self._transfer_wire(epoch, st, after)
        elif self.targets:
            self._transfer_direct(epoch, st, after, version, subset)
        elif self._writes_nothing:        # rank 0 arms every worker even when it sends nothing itself
            self._arm_and_check(epoch)
        self.epoch = epoch
        st.marks["end"] = time.perf_counter()
        st.host_ms = (st.marks["end"] - t0) * 1e3
        self.history.append(st)
        if len(self.history) > 256:
            del self.history[:128]
        return st

    def _arm_and_check(self, epoch: int) -> None:
        """Rank 0 arms the workers and fails the epoch if that did not reach all of them."""
        if self.rank != 0:
            return
        arm = self._arm(epoch)
        if arm is not None:
            arm.join()
        if self._arm_error is not None:
            self._fail_epoch(epoch, self._arm_error)
            raise TransferError(self._arm_error)

    def _handshake(self, epoch: int, version: int, subset: frozenset | None, st: SyncStats) -> list:
        """Rank 0 tags the epoch (wire modes) and arms the workers; every rank waits until its
        targets are ready.  Returns the targets' ready values (their binding generations)."""
        cfg, sess = self.config, self.session
        if self.rank == 0 and cfg.mode in WIRE_MODES:     # no done keys there: the tag has its own,
            dg = self._publish_subset(subset)              # with the entry subset the receivers cut by
            sess.set(f"ver/{epoch}", f"{version}|{dg}")
            if epoch > 16:
                sess.delete(f"ver/{epoch - 16}")
        arm = self._arm(epoch) if self.rank == 0 else None
        t1 = time.perf_counter()
        try:
            with nvtx_range("wbridge.send/ready"):
                what = f"receivers {sorted(self.targets)} to be ready for epoch {epoch}"
                keys = [f"ready/{r}/{epoch}" for r in self.targets]
                if self._board is not None:
                    b = self._board
                    b.wait([b.ready_slot(r) for r in self.targets], epoch, cfg.sync_timeout_s,
                           lambda: sess.raise_posted_error(keys), what)
                    ready = [str(b.read(b.ready_slot(r), 2)[1]).encode() for r in self.targets]
                else:
                    ready = sess.wait_checked(keys, cfg.sync_timeout_s, what)
        except (SessionTimeout, PeerError) as e:
            self._fail_epoch(epoch, str(e))
            raise TransferError(str(e)) from None
        st.wait_ready_ms = (time.perf_counter() - t1) * 1e3
        if arm is not None:
            arm.join()
        if self.rank == 0 and self._arm_error is not None:
            self._fail_epoch(epoch, self._arm_error)
            raise TransferError(self._arm_error)
        return ready

    def _prepare(self, state_dict, subset: frozenset | None, ready: list, epoch: int) -> None:
        """Make the program (or wire set) of these tensors and this subset current, opening
        the memory of workers that bound new tensors first."""
        try:
            if self.config.mode in WIRE_MODES:
                key = self._key(state_dict)
                if self._program_key != key:
                    self._wire_sets.clear()
                    self._program_key = key
                self._select_wire(state_dict, subset)
            else:
                if self._resolve_bindings(dict(zip(self.targets, ready))):
                    self._progs.clear()
                    self._program_key = None
                self._select(state_dict, subset)
        except Exception as e:
            self._fail_epoch(epoch, f"{type(e).__name__}: {e}")
            raise

    def _exchange_split_amax(self, epoch: int, st: SyncStats, after: Any) -> None:
        """Split fp8 blocks: the amax of every piece, exchanged with the blocks' co-owners."""
        try:
            tx = time.perf_counter()
            src = self._wires if self.config.mode in WIRE_MODES else self._program
            stream = None
            if src.device.type == "cuda":     # the amax pass reads what the caller's work wrote
                stream = self._stream
                self._wait_after(stream, after, src.device)
            src.set_piece_amax(self._split_amax(epoch, src.piece_amax(stream)))
            st.exchange_ms = (time.perf_counter() - tx) * 1e3
        except (SessionTimeout, PeerError, ValueError) as e:
            self._fail_epoch(epoch, str(e))
            raise TransferError(str(e)) from None

    def _transfer_wire(self, epoch: int, st: SyncStats, after: Any) -> None:
        """Wire modes: pack and send every chunk (device tensors: pack launches and NCCL sends
        ordered on the transfer stream)."""
        ws = self._wires
        if ws.device.type == "cuda":
            e0, e1 = self._ev
            with torch.cuda.stream(self._stream):
                self._wait_after(self._stream, after, ws.device)
                e0.record(self._stream)
                ws.send(self._pg, epoch, self._stream)
                e1.record(self._stream)
            e1.synchronize()
            st.device_ms = e0.elapsed_time(e1)
        else:
            ws.send(self._pg, epoch)
        st.bytes_read = ws.bytes_read
        st.bytes_written = ws.bytes_on_wire

    def _transfer_direct(self, epoch: int, st: SyncStats, after: Any, version: int,
                         subset: frozenset | None) -> None:
        """gpu_direct / nvls: launch the push program, publish completion (with the tag and
        the subset), and in the pull direction wait until every target has pulled."""
        cfg, sess = self.config, self.session
        prog = self._program
        pushed = prog is not None and len(prog.tables) > 0
        if pushed and prog.device.type == "cpu":
            t2 = time.perf_counter()
            prog.launch(epoch)
            st.device_ms = (time.perf_counter() - t2) * 1e3
        elif pushed:
            self._wait_after(self._stream, after, prog.device)
            e0, e1 = self._ev
            with nvtx_range("wbridge.send/transfer"):
                e0.record(self._stream)
                prog.launch(epoch, self._stream)
                e1.record(self._stream)
                e1.synchronize()
            st.device_ms = e0.elapsed_time(e1)
            st.status = prog.read_status()
        elif torch.cuda.is_available():
            (after if after is not None else torch.cuda.current_stream()).synchronize()   # the receivers
            # pull: the parameters must be final
        st.marks["synced"] = time.perf_counter()
        if prog is not None:
            st.bytes_read, st.bytes_written = prog.bytes_read, prog.bytes_written
        elif self.direction == "pull":     # the workers move this sender's bytes
            st.bytes_read = st.bytes_written = self._overlap_bytes(subset)
        dg = self._publish_subset(subset) if self.rank == 0 else (_digest(sorted(subset))[:16] if subset else "")
        if self._board is not None:
            b = self._board
            for r in self.targets:
                b.publish(b.done_slot(self.rank, r), [st.status, self._bind_version, int(pushed), version,
                                                      digest_word(dg)], epoch)
        else:
            done = f"{st.status}:{self._bind_version}:{int(pushed)}:{version}:{dg}"
            sess.multi_set([f"done/{self.rank}/{r}/{epoch}" for r in self.targets], [done] * len(self.targets))
        st.marks["done"] = time.perf_counter()
        if self._writes_nothing:          # pulling: the workers find this done the moment they are armed
            self._arm_and_check(epoch)
            st.marks["armed"] = time.perf_counter()
        if st.status:
            prog.clear_status()
            raise TransferError(f"transfer kernel reported status {st.status:#x} at epoch {epoch}")
        if self.direction == "pull":
            # parameters stay untouched until every target has pulled its share
            try:
                what = f"receivers {sorted(self.targets)} to pull epoch {epoch}"
                keys = [f"pulled/{r}/{epoch}" for r in self.targets]
                if self._board is not None:
                    b = self._board
                    b.wait([b.pulled_slot(r) for r in self.targets], epoch, cfg.sync_timeout_s,
                           lambda: sess.raise_posted_error(keys), what)
                    vals = [str(b.read(b.pulled_slot(r), 2)[1]).encode() for r in sorted(self.targets)]
                else:
                    vals = sess.wait_checked(keys, cfg.sync_timeout_s, what)
            except (SessionTimeout, PeerError) as e:
                raise TransferError(str(e)) from None
            bad = {r: int(v) for r, v in zip(sorted(self.targets), vals) if int(v)}
            if bad:
                raise TransferError(f"receivers reported pull status {bad} at epoch {epoch}")

def _uncovered(rmetas: dict[int, WeightData], covered: dict[tuple[int, str], int]) -> dict[int, list[str]]:
    """Per worker, the entries (scales aside) whose shards the senders' overlaps do not fill
    (``covered``: elements written, counted per destination shard)."""
    out: dict[int, list[str]] = {}
    for r, meta in rmetas.items():
        for n, shards, _dt in meta:
            if (meta.quant(n) or {}).get("role") == "scale":
                continue
            if covered.get((r, n), 0) < sum(shard_numel(sh) for sh in shards):
                out.setdefault(r, []).append(n)
    return out


def _digest(obj) -> str:
    import hashlib
    import json
    return hashlib.sha256(json.dumps(obj, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _phys_extents(pb: PhysBinding) -> list[tuple[int, int]]:
    """Byte extents of absolute-address bound shards (host receivers in this process)."""
    out = []
    for name, shards in pb.entries.items():
        es = pb.meta.dtype(name).itemsize
        for p in shards:
            span = sum((r - l - 1) * st for (l, r, _w), st in zip(p.shard, p.strides)) + 1
            out.append((p.offset, p.offset + span * es))
    return out


def _check_flag(addr: int, ranges) -> None:
    addr &= ~1                          # bit 0 marks a multicast address
    if not any(lo <= addr and addr + 8 <= hi for lo, hi in ranges):
        raise PlanBoundsError(f"flag word {addr:#x} outside the receiver's registered memory")


def session_direction(cfg: TransferConfig, receiver_metas) -> str:
    """Who runs the copy program of a ``gpu_direct`` session: ``pull`` (each receiver loads its
    copies from the senders' exported memory; the fastest way over NVLink measured here) when
    asked for and no receiver holds block-quantised (fp8) entries; otherwise ``push`` (each sender
    stores, fusing the quantisation, which halves the bytes on the link).  A session with fp8
    entries pushes everything: pulling the plain copies would only start once the quantised
    blocks are stored, after the push kernel."""
    if cfg.mode != "gpu_direct" or cfg.direction != "pull":
        return "push"
    if any(m.quant(n) for m in receiver_metas for n in m.names()):
        return "push"
    return "pull"


def wire_group(mode: str, sess: Session, rank: int, world: int, timeout_s: float, address: str):
    """The payload process group of a wire mode: gloo (host tensors) or NCCL (device tensors),
    separate from the trainer's own groups and built on the session store."""
    if mode == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts._timeout = timedelta(seconds=timeout_s)
        return dist.ProcessGroupNCCL(dist.PrefixStore("nccl", sess.store), rank, world, opts)
    return gloo_group(sess, rank, world, timeout_s, address)


def gloo_group(sess: Session, rank: int, world: int, timeout_s: float, address: str):
    """A gloo process group over the session store, separate from the trainer's groups."""
    opts = dist.ProcessGroupGloo._Options()
    opts._timeout = timedelta(seconds=timeout_s)
    ifname = os.environ.get("GLOO_SOCKET_IFNAME")
    dev = (dist.ProcessGroupGloo.create_device(interface=ifname) if ifname
           else dist.ProcessGroupGloo.create_device(hostname=address))
    opts._devices = [dev]
    return dist.ProcessGroupGloo(dist.PrefixStore("gloo", sess.store), rank, world, opts)


def _round_robin(lens: list[int]) -> np.ndarray:
    """Order taking one row from each of the concatenated parts (of ``lens`` rows) in turn."""
    k = len(lens)
    keys = np.concatenate([np.arange(n, dtype=np.int64) * k + i for i, n in enumerate(lens)]) if lens else \
        np.zeros(0, np.int64)
    return np.argsort(keys, kind="stable")


def _interleave(parts: list[Tables]) -> Tables:
    """Concatenate per-peer tables, dealing the copy items and the quantised blocks round-robin
    across the peers, so the CTAs running at any moment reach every peer: senders whose work
    for peer 0 comes first would otherwise all meet at peer 0's link, then at peer 1's, ...
    (split-block pieces keep their order: their positions index the exchanged amax)."""
    if len(parts) <= 1:
        return Tables.concat(parts)
    merged = Tables.concat(parts)
    merged.items = merged.items[_round_robin([len(p.items) for p in parts])]
    merged.qwork = merged.qwork[_round_robin([len(p.qwork) for p in parts])]
    return merged
