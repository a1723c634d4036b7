"""CUDA IPC export/import of a receiver's parameter memory.

A receiver exports every allocation that holds one of its bound tensors (found with
``cuMemGetAddressRange``, deduplicated by base address) as a CUDA IPC handle and publishes
``(allocation, offset)`` for each tensor.  A sender in another process opens each handle
once and resolves destination addresses as ``base + offset``; the transfer kernel then
stores straight into the receiver's parameters over NVLink (or into the same GPU's memory
when colocated).  A sender in the receiver's own process uses the addresses directly.
"""
from __future__ import annotations

import threading

import torch

from ..control.protocol import b64, unb64
from ..ops._ext import ext

_OPEN: dict[bytes, list] = {}     # handle -> [ptr, refs]
_OPEN_LOCK = threading.Lock()


class ExportTable:
    """Allocations backing a set of device tensors, with their IPC handles."""

    def __init__(self, device: torch.device):
        self.device = device
        self.allocs: list[dict] = []
        self._by_base: dict[int, int] = {}

    def locate(self, ptr: int) -> tuple[int, int]:
        base, size = ext().addr_range(ptr)
        idx = self._by_base.get(base)
        if idx is None:
            try:
                handle = ext().ipc_handle(base)
            except RuntimeError as e:
                raise RuntimeError(
                    f"cannot export receiver memory at {ptr:#x} through CUDA IPC ({e}); tensors from "
                    "PyTorch's expandable segments need the VMM pool (weightbridge_b200.parallel.vmm)") from None
            idx = len(self.allocs)
            self.allocs.append({"base": base, "size": size, "handle": handle})
            self._by_base[base] = idx
        return idx, ptr - base

    def to_json(self) -> list[dict]:
        return [{"base": a["base"], "size": a["size"], "handle": b64(a["handle"])} for a in self.allocs]


class ImportTable:
    """Base addresses of a peer's exported allocations in this process."""

    def __init__(self, allocs: list[dict], same_process: bool):
        self.same_process = same_process
        self.bases: list[int] = []
        self._handles: list[bytes] = []
        self._pools = []
        for a in allocs:
            if same_process:
                self.bases.append(int(a["base"]))
                continue
            if a.get("vmm"):
                # a VMM pool served as a file descriptor by the receiver process
                import os
                from .fdpass import fetch_fd
                from .vmm import ImportedPool
                fd = fetch_fd(a["fd_addr"], a["key"])
                try:
                    pool = ImportedPool(fd, int(a["size"]), torch.cuda.current_device())
                finally:
                    os.close(fd)
                self._pools.append(pool)
                self.bases.append(pool.ptr)
                continue
            h = unb64(a["handle"])
            with _OPEN_LOCK:
                ent = _OPEN.get(h)
                if ent is None:
                    ent = [ext().ipc_open(h), 0]
                    _OPEN[h] = ent
                ent[1] += 1
            self._handles.append(h)
            self.bases.append(ent[0])

    def base(self, alloc: int) -> int:
        if alloc < 0:
            return 0
        return self.bases[alloc]

    def close(self) -> None:
        for pool in self._pools:
            pool.close()
        self._pools = []
        with _OPEN_LOCK:
            for h in self._handles:
                ent = _OPEN.get(h)
                if ent is None:
                    continue
                ent[1] -= 1
                if ent[1] == 0:
                    try:
                        ext().ipc_close(ent[0])
                    finally:
                        del _OPEN[h]
        self._handles.clear()
