"""VMM parameter pools: one ``cuMemCreate`` allocation holding a rank's parameters.

A receiver that wants NVLink multicast fan-out allocates its parameters from a ``VmmPool``:
the pool can be exported as a POSIX file descriptor (other processes map it for unicast
stores) and bound to a multicast object (one ``multimem.st`` reaches every replica).  The
caching allocator's memory can do neither, which is why the pool exists.

The pool is exposed to PyTorch as a ``uint8`` tensor through ``__cuda_array_interface__``;
tensors carved from it do not own the memory, so the pool must outlive them.  The last
``tail_bytes`` of the pool are reserved for the receiver's epoch flag words.
"""
from __future__ import annotations

import threading

import torch

from ..ops._ext import ext

_POOLS: dict[int, "VmmPool"] = {}       # base address -> pool (for lookup by pointer)
_LOCK = threading.Lock()


class _CudaBuffer:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def tensor_from_ptr(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """A non-owning uint8 tensor over device memory at ``ptr``."""
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaBuffer(ptr, nbytes), device=device)


def round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


class VmmPool:
    def __init__(self, nbytes: int, device: torch.device | int, tail_bytes: int = 4096):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device_index = dev
        gran = max(ext().vmm_granularity(dev, False), ext().vmm_granularity(dev, True))
        self.tail_bytes = round_up(tail_bytes, 256)
        size = round_up(nbytes + self.tail_bytes, gran)
        self.ptr, self.size, self.handle = ext().vmm_alloc(size, dev)
        self.tensor = tensor_from_ptr(self.ptr, self.size, self.device)
        self.tensor.zero_()
        with _LOCK:
            _POOLS[self.ptr] = self

    @property
    def usable_bytes(self) -> int:
        return self.size - self.tail_bytes

    def params_buffer(self) -> torch.Tensor:
        return self.tensor[: self.usable_bytes]

    def tail(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.tail_bytes:
            raise ValueError(f"pool tail holds {self.tail_bytes} bytes, {nbytes} requested")
        return self.tensor[self.usable_bytes:self.usable_bytes + nbytes]

    def export_fd(self) -> int:
        return ext().vmm_export_fd(self.handle)

    def contains(self, ptr: int) -> bool:
        return self.ptr <= ptr < self.ptr + self.size

    def free(self) -> None:
        """Unmap and release; every tensor carved from the pool must be dead."""
        with _LOCK:
            _POOLS.pop(self.ptr, None)
        self.tensor = None
        ext().vmm_free(self.ptr, self.size, self.handle)


def find_pool(ptr: int) -> VmmPool | None:
    with _LOCK:
        for p in _POOLS.values():
            if p.contains(ptr):
                return p
    return None


class ImportedPool:
    """A peer's VMM pool mapped into this process (unicast stores, e.g. flag words)."""

    def __init__(self, fd: int, size: int, device: torch.device | int):
        dev = device if isinstance(device, int) else (torch.device(device).index or 0)
        self.ptr, self.size, self.handle = ext().vmm_import_fd(fd, size, dev)

    def close(self) -> None:
        ext().vmm_free(self.ptr, self.size, self.handle)
