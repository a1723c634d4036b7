"""Per-sync handshake words in shared memory for a session whose peers share one host.

``gpu_direct`` and ``nvls`` need every sender and worker on one node, so the per-sync
notifications - a worker's ``ready`` (it is idle; in the push direction the senders may now
store into it), a sender's ``done`` (its kernel finished, or in the pull direction its
parameters are final) and a worker's ``pulled`` - are words in one shared-memory file instead
of session-store keys: a notification is a store of a few words ended by a release store of the
epoch, and a wait polls the epoch words (``csrc/wb_board.cpp``: spinning, then yielding the
core between polls, with the GIL released) instead of a TCP round trip to the store.  Errors
still travel through the session store: a waiter checks the store keys of the notifications it
waits for every few milliseconds, so an error a peer (or the liveness watcher) posted there
ends the wait as before.

Layout (int64 words): an 8-word header, then one 8-word slot per worker for ``ready``
(epoch, binding generation), one per worker for ``pulled`` (epoch, status), and one per
(sender, worker) pair for ``done`` (epoch, status, sender memory version, pushed, version tag,
subset digest).  Workers are indexed by their global rank minus the sender count.
"""
from __future__ import annotations

import mmap
import os
import tempfile
import time
from typing import Callable

import numpy as np

from ..ops._ext import ext
from .session import SessionTimeout

_HEADER, _SLOT = 8, 8
_MAGIC = 0x5742424F415244      # "WBBOARD"
_POLL_NS = 5_000_000           # store check between bounded waits


def board_dir() -> str:
    return "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()


def digest_word(dg: str) -> int:
    """A subset digest (up to 16 hex characters, "" for every entry) as a signed 64-bit word."""
    if not dg:
        return 0
    v = int(dg[:16], 16)
    return v - (1 << 64) if v >= 1 << 63 else v


def word_digest(v: int) -> str:
    return format(v & ((1 << 64) - 1), "016x") if v else ""


class SyncBoard:
    def __init__(self, path: str, n_senders: int, n_workers: int, create: bool = False):
        self.path, self.W, self.M = path, int(n_senders), int(n_workers)
        words = _HEADER + _SLOT * (2 * self.M + self.W * self.M)
        size = 8 * words
        if create:
            fd = os.open(path, os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
            try:
                os.ftruncate(fd, size)
            except OSError:
                os.close(fd)
                os.unlink(path)
                raise
        else:
            fd = os.open(path, os.O_RDWR)
        try:
            self._mm = mmap.mmap(fd, size)
        finally:
            os.close(fd)
        self._words = np.frombuffer(self._mm, dtype=np.int64)
        self.base = int(self._words.ctypes.data)
        if create:
            self._words[:3] = (_MAGIC, self.W, self.M)
        elif tuple(int(x) for x in self._words[:3]) != (_MAGIC, self.W, self.M):
            raise ValueError(f"{path} is not this session's handshake board")
        self._owner = create
        if create:                     # the file outlives a process that never closes the board
            import atexit
            atexit.register(self.close)

    @staticmethod
    def create(session_id: str, n_senders: int, n_workers: int) -> "SyncBoard":
        return SyncBoard(os.path.join(board_dir(), f"wbridge-board-{session_id}"), n_senders, n_workers, create=True)

    def describe(self) -> dict:
        return {"path": self.path, "senders": self.W, "workers": self.M}

    @staticmethod
    def attach(desc: dict | None) -> "SyncBoard | None":
        if not desc:
            return None
        return SyncBoard(desc["path"], desc["senders"], desc["workers"])

    # -- slots ---------------------------------------------------------------------------
    def ready_slot(self, r: int) -> int:
        return _HEADER + _SLOT * (r - self.W)

    def pulled_slot(self, r: int) -> int:
        return _HEADER + _SLOT * (self.M + r - self.W)

    def done_slot(self, s: int, r: int) -> int:
        return _HEADER + _SLOT * (2 * self.M + s * self.M + (r - self.W))

    def publish(self, slot: int, fields: list[int], epoch: int) -> None:
        ext().board_publish(self.base, slot, [int(f) for f in fields], int(epoch))

    def read(self, slot: int, n: int) -> list[int]:
        return ext().board_read(self.base, slot, n)

    def wait(self, slots: list[int], epoch: int, timeout_s: float, check: Callable[[], None], what: str) -> None:
        """Until every slot holds ``epoch`` (or a later one); ``check`` runs between bounded
        waits and raises if a peer posted an error; ``SessionTimeout`` after ``timeout_s``."""
        if not slots:
            return
        deadline = time.monotonic() + timeout_s
        while True:
            left = deadline - time.monotonic()
            if ext().board_wait(self.base, slots, int(epoch), int(1e9 * max(0.0, min(left, _POLL_NS / 1e9)))):
                return
            check()
            if time.monotonic() >= deadline:
                raise SessionTimeout(f"timed out after {timeout_s:.1f}s waiting for {what}")

    def close(self) -> None:
        words, self._words = self._words, None
        del words
        try:
            self._mm.close()
        except (BufferError, ValueError):   # a view is still alive somewhere, or already closed
            pass
        if self._owner:
            try:
                os.unlink(self.path)
            except OSError:
                pass
            self._owner = False
