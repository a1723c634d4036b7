"""Chunked wire transfers of the wire modes (``cpu_direct`` over gloo, ``nccl``).

Each (sender, receiver) pair's overlap is cut into chunks of whole entries
(``core/wire.py``).  Per peer a side holds two buffers of the largest chunk and one work
table per chunk: the sender packs chunk k into buffer k % 2 while chunk k - 1 is on the wire
and, before packing chunk k + 2 into the same buffer, waits for chunk k's send; the receiver
keeps two receives posted per peer and unpacks each chunk as it lands.  Device tensors
(``nccl``) pack and unpack with one transfer-kernel launch per chunk, and ``work.wait()``
only orders streams; host tensors (``cpu_direct``) use the C++ executor.

Parity: the reference sends one buffer of the whole overlap per pair, packed on the host
(``wbridge/backend/direct_sender.py:184-198``, ``wbridge/frontend/receiver.py:217-230``).
"""
from __future__ import annotations

import numpy as np
import torch

from ..core.plan import Tables, lower_ops, plan_pair, storage_ranges, validate_tables, wire_binding
from ..core.shard import WeightData
from ..core.wire import buffer_bytes, wire_chunks

_ABS = lambda _alloc: 0     # noqa: E731  (wire and local bindings hold absolute addresses)


def chunk_tag(epoch: int, k: int) -> int:
    """Message tag of chunk ``k`` of sync ``epoch`` (gloo matches tags; NCCL ignores them)."""
    return ((epoch & 0x7FFF) << 16) | (k & 0xFFFF)


class WireSet:
    """One side's chunked wires: per peer, the buffers and ``(tables, buffer, nbytes)`` per chunk."""

    def __init__(self, device: torch.device):
        self.device = device
        self.peers: dict[int, tuple[list[torch.Tensor], list[tuple[Tables, int, int]]]] = {}
        self.progs: dict[int, list] = {}
        self.amax_prog = None
        self._amax = np.zeros(0, dtype=np.float32)

    # -- construction --------------------------------------------------------------------
    def _buffers(self, peer: int, overlap: WeightData, chunks: list[WeightData], chunk_bytes: int,
                 shared: dict[int, list[torch.Tensor]] | None) -> list[torch.Tensor]:
        """Two buffers (one for a single chunk) that hold any chunk of ``overlap`` or of a
        subset of it, so the wire sets of partial syncs reuse the full set's (``shared``)."""
        n = min(2, len(chunks))
        need = max(c.total_nbytes() for c in chunks)
        have = (shared or {}).get(peer)
        if have is not None and len(have) >= n and all(b.numel() >= need for b in have[:n]):
            return have[:n]
        size = max(need, buffer_bytes(overlap, chunk_bytes))
        return [torch.empty(size, dtype=torch.uint8, device=self.device) for _ in range(n)]

    def buffers(self) -> dict[int, list[torch.Tensor]]:
        return {p: bufs for p, (bufs, _items) in self.peers.items()}

    @staticmethod
    def for_sender(sphys, overlaps: dict[int, WeightData], targets: dict[int, list[str]], device, cfg,
                   src_ranges, shared: dict[int, list[torch.Tensor]] | None = None) -> "WireSet":
        """``shared``: per peer, buffers of another wire set of the same peers (the full sync's,
        when this one is a partial sync) to reuse where they are large enough."""
        ws = WireSet(device)
        for r, names in sorted(targets.items()):
            chunks = wire_chunks(overlaps[r], cfg.wire_chunk_bytes)
            if not chunks:
                continue
            bufs = ws._buffers(r, overlaps[r], chunks, cfg.wire_chunk_bytes, shared)
            items = []
            for k, ov in enumerate(chunks):
                b = k % len(bufs)
                t = lower_ops(plan_pair(sphys, wire_binding(ov, base=bufs[b].data_ptr()), names=names, overlap_meta=ov),
                              _ABS, _ABS, item_bytes=cfg.item_bytes, receiver=r)
                if cfg.validate_plan:
                    validate_tables(t, src_ranges, storage_ranges([bufs[b]]))
                items.append((t, b, ov.total_nbytes()))
            ws.peers[r] = (bufs, items)
        ws._programs(cfg, pieces=True)
        return ws

    @staticmethod
    def for_receiver(rphys, overlaps: dict[int, WeightData], device, cfg, dst_ranges, chunk_bytes: int,
                     shared: dict[int, list[torch.Tensor]] | None = None) -> "WireSet":
        """``chunk_bytes`` is the senders' (the session carries it), so both sides cut alike."""
        ws = WireSet(device)
        for s, ov_all in sorted(overlaps.items()):
            chunks = wire_chunks(ov_all, chunk_bytes)
            if not chunks:
                continue
            bufs = ws._buffers(s, ov_all, chunks, chunk_bytes, shared)
            items = []
            for k, ov in enumerate(chunks):
                b = k % len(bufs)
                t = lower_ops(plan_pair(wire_binding(ov, base=bufs[b].data_ptr()), rphys), _ABS, _ABS,
                              item_bytes=cfg.item_bytes)
                if cfg.validate_plan:
                    validate_tables(t, storage_ranges([bufs[b]]), dst_ranges)
                items.append((t, b, ov.total_nbytes()))
            ws.peers[s] = (bufs, items)
        ws._programs(cfg, pieces=False)
        return ws

    def _programs(self, cfg, pieces: bool) -> None:
        self._all = Tables.concat([t for p in sorted(self.peers) for t, _b, _n in self.peers[p][1]])
        if self.device.type != "cuda":
            self._amax = np.zeros(len(self.all_tables.pieces), dtype=np.float32)
            return
        from ..ops.executor import LaunchConfig, TransferProgram
        lc = LaunchConfig(mode=cfg.kernel_mode, piece_bytes=cfg.piece_bytes, grid=cfg.grid or None)
        self.progs = {p: [TransferProgram(t, self.device, [], lc) for t, _b, _n in items]
                      for p, (_bufs, items) in self.peers.items()}
        allp = self.all_tables.pieces
        if pieces and len(allp):       # the amax pass of split fp8 blocks reads only the sources
            empty = Tables.empty()
            self.amax_prog = TransferProgram(Tables(empty.items, empty.qdescs, empty.qwork, pieces=allp),
                                             self.device, [], lc)

    # -- bookkeeping ---------------------------------------------------------------------
    @property
    def all_tables(self) -> Tables:
        """Every chunk's tables, peers in ascending order, chunks in order (the piece order)."""
        return self._all

    @property
    def bytes_on_wire(self) -> int:
        return sum(n for _bufs, items in self.peers.values() for _t, _b, n in items)

    @property
    def bytes_read(self) -> int:
        return sum(t.bytes_read for _bufs, items in self.peers.values() for t, _b, _n in items)

    @property
    def n_chunks(self) -> int:
        return sum(len(items) for _bufs, items in self.peers.values())

    # -- split fp8 blocks ------------------------------------------------------------------
    def piece_amax(self, stream=None) -> np.ndarray:
        if self.amax_prog is not None:
            return self.amax_prog.piece_amax(stream)
        from ..ops.executor import cpu_piece_amax
        return cpu_piece_amax(self.all_tables)

    def set_piece_amax(self, values: np.ndarray) -> None:
        values = np.asarray(values, dtype=np.float32)
        self._amax = values.copy()
        if self.progs:
            first = 0
            for p in sorted(self.peers):
                for prog in self.progs[p]:
                    if prog.n_pieces:
                        prog.set_piece_amax(values[first:first + prog.n_pieces])
                        first += prog.n_pieces

    def _host_amax_slices(self) -> dict[tuple[int, int], np.ndarray | None]:
        out, first = {}, 0
        for p in sorted(self.peers):
            for k, (t, _b, _n) in enumerate(self.peers[p][1]):
                n = len(t.pieces)
                out[(p, k)] = self._amax[first:first + n] if n else None
                first += n
        return out

    # -- transfers -----------------------------------------------------------------------
    def send(self, pg, epoch: int, stream: torch.cuda.Stream | None = None) -> None:
        """Pack and send every chunk to every peer (device tensors: call inside
        ``torch.cuda.stream(stream)``; returns once everything is enqueued and, for host
        tensors, sent)."""
        from ..ops.executor import cpu_execute
        order = sorted(self.peers)
        works: dict[int, list] = {p: [] for p in order}
        amax = self._host_amax_slices() if not self.progs else None
        for k in range(max((len(self.peers[p][1]) for p in order), default=0)):
            for p in order:
                bufs, items = self.peers[p]
                if k >= len(items):
                    continue
                t, b, n = items[k]
                if k >= 2:
                    works[p][k - 2].wait()       # its buffer is about to be packed again
                if self.progs:
                    self.progs[p][k].launch(epoch, stream, signal=False)
                else:
                    cpu_execute(t, amax[(p, k)])
                works[p].append(pg.send([bufs[b][:n]], p, chunk_tag(epoch, k)))
        for p in order:                          # each work is waited once: a second wait of a
            for w in works[p][-2:]:              # gloo send waits for another completion
                w.wait()

    def recv(self, pg, epoch: int, stream: torch.cuda.Stream | None = None) -> None:
        """Receive and unpack every chunk from every peer, two receives posted per peer."""
        from ..ops.executor import cpu_execute
        order = sorted(self.peers)
        works: dict[int, dict[int, object]] = {p: {} for p in order}

        def post(p: int, k: int) -> None:
            bufs, items = self.peers[p]
            _t, b, n = items[k]
            works[p][k] = pg.recv([bufs[b][:n]], p, chunk_tag(epoch, k))

        for p in order:
            for k in range(min(2, len(self.peers[p][1]))):
                post(p, k)
        for k in range(max((len(self.peers[p][1]) for p in order), default=0)):
            for p in order:
                items = self.peers[p][1]
                if k >= len(items):
                    continue
                works[p][k].wait()
                if self.progs:
                    self.progs[p][k].launch(epoch, stream, signal=False)
                else:
                    cpu_execute(items[k][0])
                if k + 2 < len(items):
                    post(p, k + 2)                # after the unpack that frees its buffer
