"""Launchers for the work tables: the sm_100a transfer kernel and the C++ CPU executor.

``TransferProgram`` keeps one sender's tables resident on its GPU (uploaded once at
connect), plus the completion state of the launch: a scratch counter, the table of flag
addresses the last CTA publishes to, the epoch word (copied host->device from pinned
memory on every sync) and a status word.  A sync is then a single kernel launch.
"""
from __future__ import annotations

import logging
import os
from dataclasses import dataclass

import numpy as np
import torch

from ..core.plan import OP_COPY, Tables
from ._ext import ext

logger = logging.getLogger(__name__)

# TMA pipeline modes of the kernel (stages x piece bytes of shared memory per CTA).  In the
# TMA modes the same shared memory is also the ring of quant stages (32 KiB blocks loaded by
# tensor-map copies).  MODE_AUTO: MODE_BULK8 for copy-only programs (one CTA per SM keeps the
# most bytes in flight per CTA: 1.016 of the measured HBM copy, against 0.963 with BULK4);
# BULK4 for programs with quant blocks (three CTAs per SM, two quant stages each: quantising
# 0.949, quant + copies 0.955, against 0.916 / 0.875 on the vector path and 0.497 with BULK8,
# where eight warps per SM cannot hide the quantiser's barriers).  A program with nothing for
# the TMA engine launches in vector mode.
MODE_AUTO, MODE_VECTOR, MODE_BULK8, MODE_BULK12, MODE_BULK4 = -1, 0, 1, 2, 3
AUTO_QUANT_MODE = MODE_BULK4
DEFAULT_SPIN_LIMIT = 1 << 26


def _np_to_tensor(a: np.ndarray, device) -> torch.Tensor:
    if len(a) == 0:
        return torch.zeros(16, dtype=torch.uint8, device=device)
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).copy())
    return t.to(device)


def bulk_eligible(items: np.ndarray) -> np.ndarray:
    """Items the TMA pipeline may move: plain copies, 16-byte aligned everywhere."""
    bits = (items["src"] | items["dst"] | items["src_pitch"].astype(np.uint64)
            | items["dst_pitch"].astype(np.uint64) | items["row_bytes"].astype(np.uint64))
    return ((items["op"] & 0xFF) == OP_COPY) & ((bits & np.uint64(15)) == 0)


def cpu_execute(tables: Tables, piece_amax: np.ndarray | None = None) -> None:
    """Run work tables on the host (addresses are host pointers).  Split-block pieces are
    quantised with ``piece_amax`` (one block amax per piece), which they need."""
    if len(tables.pieces):
        if piece_amax is None or len(piece_amax) != len(tables.pieces):
            raise ValueError("split-block pieces need their block amax (one value per piece)")
        pc = np.ascontiguousarray(tables.pieces)
        am = np.ascontiguousarray(piece_amax, dtype=np.float32)
        ext().cpu_split_quant(pc.ctypes.data, len(pc), am.ctypes.data)
    it = np.ascontiguousarray(tables.items)
    qd = np.ascontiguousarray(tables.qdescs)
    qw = np.ascontiguousarray(tables.qwork)
    ext().cpu_execute(it.ctypes.data if len(it) else 0, len(it), qd.ctypes.data if len(qd) else 0,
                      qw.ctypes.data if len(qw) else 0, len(qw))


def cpu_piece_amax(tables: Tables) -> np.ndarray:
    """Split blocks, first step on the host: max |x| over every piece."""
    out = np.zeros(len(tables.pieces), dtype=np.float32)
    if len(out):
        pc = np.ascontiguousarray(tables.pieces)
        ext().cpu_split_amax(pc.ctypes.data, len(pc), out.ctypes.data)
    return out


@dataclass
class LaunchConfig:
    mode: int = MODE_AUTO
    piece_bytes: int = 16384
    grid: int | None = None
    spin_limit: int = DEFAULT_SPIN_LIMIT

    @staticmethod
    def from_env() -> "LaunchConfig":
        c = LaunchConfig()
        c.mode = int(os.environ.get("WBRIDGE_KERNEL_MODE", c.mode))
        c.piece_bytes = int(os.environ.get("WBRIDGE_PIECE_BYTES", c.piece_bytes))
        g = os.environ.get("WBRIDGE_GRID")
        c.grid = int(g) if g else None
        return c


class TransferProgram:
    """Device-resident tables of one sender plus its completion signal."""

    def __init__(self, tables: Tables, device: torch.device | int | str,
                 flag_addrs: list[int] | None = None, config: LaunchConfig | None = None,
                 local_flag: bool = False):
        """``local_flag``: the launch also publishes its epoch to a word of this program, next
        to the status word, so one read returns both (``read_status_and_flag``)."""
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        self.config = config or LaunchConfig.from_env()
        if self.config.mode == MODE_AUTO:
            from dataclasses import replace
            self.config = replace(self.config, mode=AUTO_QUANT_MODE if len(tables.qwork) else MODE_BULK8)
        self.tables = tables
        items = tables.items
        if self.config.mode != MODE_VECTOR and len(items):
            mask = bulk_eligible(items)
            self.bulk_np, self.items_np = items[mask], items[~mask]
        else:
            self.bulk_np, self.items_np = items[:0], items
        dev = self.device
        self.items = _np_to_tensor(self.items_np, dev)
        self.bulk = _np_to_tensor(self.bulk_np, dev)
        self.qdescs = _np_to_tensor(tables.qdescs, dev)
        self.qwork = _np_to_tensor(tables.qwork, dev)
        # TMA-fed quant blocks: a tensor map per quant matrix (TMA modes only)
        self.n_tma_quant = 0
        self.qmaps = self.qtma = None
        if self.config.mode != MODE_VECTOR and len(tables.qdescs) and len(tables.qwork):
            qd = np.ascontiguousarray(tables.qdescs)
            maps = np.zeros(len(qd) * 128, dtype=np.uint8)
            valid = np.zeros(len(qd), dtype=np.uint8)
            try:
                n_maps = ext().encode_quant_maps(qd.ctypes.data, len(qd), maps.ctypes.data, valid.ctypes.data)
            except RuntimeError as e:           # no tensor-map encoder in this driver: register path
                logger.warning("quant blocks take the register path: %s", e)
                n_maps = 0
            if n_maps:
                self.qmaps = torch.from_numpy(maps).to(dev)          # caching-allocator blocks: 512-byte aligned
                self.qtma = torch.from_numpy(valid).to(dev)
                self.n_tma_quant = int(valid[tables.qwork["desc"]].sum())
        flag_addrs = list(flag_addrs or [])
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        # [status (low 4 bytes), local flag]: one 16-byte read returns both
        self.status_flag = torch.zeros(2, dtype=torch.int64, device=dev)
        self.status = self.status_flag[:1].view(torch.int32)[:1]
        if local_flag:
            flag_addrs.append(self.status_flag[1:].data_ptr())
        self.n_flags = len(flag_addrs)
        self.flags = torch.tensor(flag_addrs or [0], dtype=torch.int64, device=dev)
        self.epoch_dev = torch.zeros(1, dtype=torch.int64, device=dev)
        self.epoch_host = torch.zeros(1, dtype=torch.int64, pin_memory=True)
        self.n_sms = ext().num_sms(dev.index if dev.index is not None else torch.cuda.current_device())
        self.launches = 0
        self.status_host = torch.zeros(2, dtype=torch.int64, pin_memory=True)
        self.launch_mode = self.config.mode if (len(self.bulk_np) or self.n_tma_quant) else MODE_VECTOR
        launch_mode = self.launch_mode
        self._fixed = (self.items.data_ptr(), len(self.items_np), self.bulk.data_ptr(), len(self.bulk_np),
                       self.qdescs.data_ptr(), self.qwork.data_ptr(), len(tables.qwork), self.config.piece_bytes,
                       self.config.spin_limit, self.counter.data_ptr(), self.flags.data_ptr() if self.n_flags else 0,
                       self.n_flags, self.epoch_dev.data_ptr(), self.status.data_ptr(), launch_mode, self.grid(),
                       self.epoch_host.data_ptr(),
                       self.qmaps.data_ptr() if self.qmaps is not None else 0,
                       self.qtma.data_ptr() if self.qtma is not None else 0)
        # split-block pieces: amax per piece (device, pinned copy) and the exchanged block amax
        self.n_pieces = len(tables.pieces)
        if self.n_pieces:
            self.pieces = _np_to_tensor(tables.pieces, dev)
            self.partial = torch.zeros(self.n_pieces, dtype=torch.float32, device=dev)
            self.amax = torch.zeros(self.n_pieces, dtype=torch.float32, device=dev)
            self.partial_host = torch.zeros(self.n_pieces, dtype=torch.float32, pin_memory=True)
            self.amax_host = torch.zeros(self.n_pieces, dtype=torch.float32, pin_memory=True)

    def piece_amax(self, stream: torch.cuda.Stream | None = None) -> np.ndarray:
        """Split blocks, first step: max |x| over every piece (launch, copy back, wait)."""
        if not self.n_pieces:
            return np.zeros(0, dtype=np.float32)
        stream = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(stream):
            ext().split_amax(self.pieces.data_ptr(), self.n_pieces, self.partial.data_ptr(), stream.cuda_stream)
            self.partial_host.copy_(self.partial, non_blocking=True)
        stream.synchronize()
        return self.partial_host.numpy().copy()

    def set_piece_amax(self, values: np.ndarray) -> None:
        """The block amax of every piece for the next launches (after the senders' exchange)."""
        self.amax_host.numpy()[:] = values

    @property
    def bytes_read(self) -> int:
        return self.tables.bytes_read

    @property
    def bytes_written(self) -> int:
        return self.tables.bytes_written

    def grid(self) -> int:
        c = self.config
        if c.grid:
            return c.grid
        work = len(self.items_np) + len(self.tables.qwork) + len(self.bulk_np)
        if self.launch_mode == MODE_VECTOR:
            per_sm = 4
        else:
            smem = ext().bulk_stages(c.mode) * c.piece_bytes
            per_sm = max(1, min(4, (200 * 1024) // max(smem, 1)))
        return max(1, min(work, self.n_sms * per_sm))

    def launch(self, epoch: int, stream: torch.cuda.Stream | None = None, signal: bool = True) -> None:
        """Copy the epoch host->device and launch the kernel on ``stream``.  With
        ``signal=False`` the launch publishes no flags (ordering is the caller's job)."""
        stream = stream or torch.cuda.current_stream(self.device)
        if self.n_pieces:           # before the transfer kernel, whose last CTA publishes the flags
            with torch.cuda.stream(stream):
                self.amax.copy_(self.amax_host, non_blocking=True)
                ext().split_quant(self.pieces.data_ptr(), self.n_pieces, self.amax.data_ptr(), stream.cuda_stream)
        # one native call: the epoch (pinned host word -> device) and the launch
        ext().transfer_launch(self._fixed, int(epoch) if signal else -1, stream.cuda_stream)
        self.launches += 1

    def read_status(self) -> int:
        return ext().read_words(self.status_flag.data_ptr(), self.status_host.data_ptr(), 1)[0] & 0xFFFFFFFF

    def read_status_and_flag(self) -> tuple[int, int]:
        """The status bits and the local flag word (``local_flag=True``), in one read."""
        v = ext().read_words(self.status_flag.data_ptr(), self.status_host.data_ptr(), 2)
        return v[0] & 0xFFFFFFFF, v[1]

    def clear_status(self) -> None:
        self.status.zero_()


class HostProgram:
    """The same work tables executed on the host by the C++ executor, with the epoch written
    to the flag words afterwards.  Runs the device protocol (tables, flags, status) when the
    sender and its receivers hold CPU tensors in one process, e.g. in CPU tests."""

    def __init__(self, tables: Tables, flag_addrs: list[int] | None = None):
        self.tables = tables
        self.flag_addrs = list(flag_addrs or [])
        self.device = torch.device("cpu")
        self.launches = 0
        self.n_pieces = len(tables.pieces)
        self._amax = np.zeros(self.n_pieces, dtype=np.float32)

    def piece_amax(self, stream=None) -> np.ndarray:
        return cpu_piece_amax(self.tables)

    def set_piece_amax(self, values: np.ndarray) -> None:
        self._amax = np.asarray(values, dtype=np.float32).copy()

    bytes_read = property(lambda self: self.tables.bytes_read)
    bytes_written = property(lambda self: self.tables.bytes_written)

    def grid(self) -> int:
        return 0

    def launch(self, epoch: int, stream=None, signal: bool = True) -> None:
        import ctypes
        cpu_execute(self.tables, self._amax)
        if signal:
            for a in self.flag_addrs:
                ctypes.c_int64.from_address(a).value = epoch
        self.launches += 1

    def read_status(self) -> int:
        return 0

    def clear_status(self) -> None:
        pass


def wait_flags(flags: torch.Tensor, epoch: torch.Tensor, timeout_s: float, status: torch.Tensor,
               where: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
    """Launch a bounded device-side wait until every flag word reaches ``epoch[0]``; on
    timeout the kernel sets ST_FLAG_TIMEOUT in ``status`` (and the first index in ``where``)
    and returns.  Only for flags written by another GPU: two kernels on one GPU that wait
    on each other have no co-scheduling guarantee."""
    stream = stream or torch.cuda.current_stream(flags.device)
    ext().wait_flags(flags.data_ptr(), flags.numel(), epoch.data_ptr(), int(timeout_s * 1e9), status.data_ptr(),
                     where.data_ptr() if where is not None else 0, stream.cuda_stream)
