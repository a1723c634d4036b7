"""NVLink multicast (NVLS) fan-out: one ``multimem.st`` writes the same bytes into every
rollout replica through the NVSwitch.

For a *replica group* (receivers with identical metadata and identical pool-relative
bindings, e.g. several SGLang TP1 replicas), sender rank 0 creates one multicast object the
size of a replica's VMM pool and shares it as a file descriptor.  Every participant adds its
device; replicas bind their pool to it; senders back it with scratch memory nobody reads
(every device added to the object must back all of it: a sender binds one window of at most
``SCRATCH_WINDOW`` bytes at every window offset, see ``McMember.bind_scratch``) and map the
object.  Stores to ``mc_base + offset`` then land at ``offset`` in every bound pool.  The transfer kernel writes
such items with ``multimem.st.relaxed.sys.global.v4.f32`` (16-byte aligned items only) and
publishes the epoch to each replica's flag word with ordinary unicast stores.

Teardown runs in a fixed order: senders unmap, then everyone unbinds and releases.  A
process that exits while its memory is still bound to the object can fault its peers, so
failure tests never use this path.

Parity: the reference re-packs and re-sends the same chunk to every replica
(``wbridge/utils/data.py:299-306``, ``wbridge/backend/direct_sender.py:193-195``).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import logging

from ..ops._ext import ext
from .fdpass import FdServer, fetch_fd
from .vmm import VmmPool

logger = logging.getLogger(__name__)


SCRATCH_WINDOW = 1 << 30          # a sender's backing of a multicast object: at most this much


def scratch_window(size: int, device: int, window: int = SCRATCH_WINDOW) -> int:
    """The largest multiple of the multicast granularity that divides ``size`` and is at most
    ``window`` (at least one granule)."""
    gran = max(ext().vmm_granularity(device, True), ext().vmm_granularity(device, False))
    if size % gran:
        return size
    n = size // gran
    best = 1
    for k in range(1, n + 1):
        if k * gran > window:
            break
        if n % k == 0:
            best = k
    return best * gran


def nvls_supported(device_index: int) -> bool:
    """Whether the device reports NVLink multicast support (a driver query that fails is
    logged and counts as no support)."""
    try:
        return bool(ext().multicast_supported(device_index))
    except Exception:
        logger.warning("multicast support query failed on device %d", device_index, exc_info=True)
        return False


def replica_groups(receivers: dict[int, dict]) -> list[list[int]]:
    """Receivers whose metadata and pool-relative physical bindings are identical (and that
    live in VMM pools of the same size) form a replica group; groups of one are dropped."""
    by_key: dict[str, list[int]] = {}
    for r, info in sorted(receivers.items()):
        pool = info.get("pool")
        if not pool:
            continue
        key = json.dumps([info["binding"], pool["size"]], sort_keys=True)
        by_key.setdefault(key, []).append(r)
    return [g for g in by_key.values() if len(g) > 1]


@dataclass
class McMember:
    """This process's share of one multicast object."""
    group: int
    size: int
    device: int
    handle: int = 0
    mapped: tuple | None = None          # (va, size, handle) when mapped
    bound: bool = False
    scratch: VmmPool | None = None
    server: FdServer | None = None
    notes: list[str] = field(default_factory=list)

    @property
    def va(self) -> int:
        return self.mapped[0] if self.mapped else 0

    def create(self, num_devices: int) -> None:
        self.handle = ext().mc_create(self.size, num_devices)
        self.server = FdServer()
        self.server.publish(f"mc{self.group}", ext().vmm_export_fd(self.handle))

    def join(self, address: str) -> None:
        fd = fetch_fd(address, f"mc{self.group}")
        try:
            self.handle = ext().mc_import_fd(fd)
        finally:
            os.close(fd)

    def add_device(self) -> None:
        ext().mc_add_device(self.handle, self.device)

    def bind(self, pool: VmmPool) -> None:
        if pool.size != self.size:
            raise ValueError(f"pool of {pool.size} bytes cannot back a {self.size}-byte multicast object")
        ext().mc_bind_mem(self.handle, 0, pool.handle, 0, self.size)
        self.bound = True

    def bind_scratch(self, window: int = SCRATCH_WINDOW) -> None:
        """Back this (sender) device's share of the object with memory nobody reads.  Every
        device added to a multicast object must back all of it, but a sender only issues the
        stores: one ``window``-sized allocation is bound at every window offset of the object
        (the multimem stores that land here overwrite each other), so the sender pays the
        window instead of a whole replica.  If the driver refuses to bind one allocation at
        several offsets, a scratch pool of the object's full size is used instead (noted)."""
        w = scratch_window(self.size, self.device, window)
        if w < self.size:
            self.scratch = VmmPool(w, self.device, tail_bytes=0)
            done = 0
            try:
                for off in range(0, self.size, w):
                    ext().mc_bind_mem(self.handle, off, self.scratch.handle, 0, w)
                    done += w
                self.bound = True
                return
            except RuntimeError as e:
                self.notes.append(f"windowed scratch refused after {done} bytes ({e}); binding {self.size} bytes")
                if done:
                    ext().mc_unbind(self.handle, self.device, 0, done)
                self.scratch.free()
                self.scratch = None
        self.scratch = VmmPool(self.size, self.device, tail_bytes=0)
        if self.scratch.size != self.size:
            raise ValueError("scratch pool size differs from the multicast object")
        self.bind(self.scratch)

    @property
    def scratch_bytes(self) -> int:
        return self.scratch.size if self.scratch is not None else 0

    def map(self) -> int:
        self.mapped = ext().mc_map(self.handle, self.size, self.device)
        return self.va

    def teardown_mapping(self) -> None:
        if self.mapped:
            ext().va_unmap(self.mapped[0], self.mapped[1])
            self.mapped = None

    def teardown_binding(self) -> None:
        if self.bound:
            ext().mc_unbind(self.handle, self.device, 0, self.size)
            self.bound = False
        if self.scratch is not None:
            self.scratch.free()
            self.scratch = None
        if self.handle:
            ext().mem_release(self.handle)
            self.handle = 0
        if self.server is not None:
            self.server.close()
            self.server = None
