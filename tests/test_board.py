"""The same-host handshake board: release/acquire words in shared memory between processes."""
import multiprocessing as mp
import os
import time

import pytest

from weightbridge_b200.control.board import SyncBoard, digest_word, word_digest
from weightbridge_b200.control.session import SessionTimeout


def _peer(desc, q):
    b = SyncBoard.attach(desc)
    try:
        b.wait([b.ready_slot(3)], 1, 10.0, lambda: None, "ready")
        q.put(("ready", b.read(b.ready_slot(3), 2)))
        b.publish(b.done_slot(1, 3), [0, 7, 1, 42, digest_word("0123456789abcdef")], 1)
    finally:
        b.close()


def test_board_round_trip_between_processes():
    b = SyncBoard.create(f"test-{os.getpid()}-{time.time_ns()}", n_senders=2, n_workers=2)
    try:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        p = ctx.Process(target=_peer, args=(b.describe(), q))
        p.start()
        b.publish(b.ready_slot(3), [5], 1)                      # worker 3 ready, binding generation 5
        b.wait([b.done_slot(1, 3)], 1, 20.0, lambda: None, "done")
        w = b.read(b.done_slot(1, 3), 6)
        assert w[:5] == [1, 0, 7, 1, 42] and word_digest(w[5]) == "0123456789abcdef"
        assert q.get(timeout=20) == ("ready", [1, 5])
        p.join(20)
        assert p.exitcode == 0
    finally:
        b.close()
    assert not os.path.exists(b.path)


def test_board_slots_are_distinct_and_waits_are_bounded():
    b = SyncBoard.create(f"test-{os.getpid()}-{time.time_ns()}", n_senders=3, n_workers=4)
    try:
        slots = [b.ready_slot(r) for r in range(3, 7)] + [b.pulled_slot(r) for r in range(3, 7)] + \
            [b.done_slot(s, r) for s in range(3) for r in range(3, 7)]
        assert len(set(slots)) == len(slots) and max(slots) + 8 <= len(b._words)
        checks = []
        t0 = time.monotonic()
        with pytest.raises(SessionTimeout):
            b.wait([b.pulled_slot(4)], 1, 0.05, lambda: checks.append(1), "pulled")
        assert time.monotonic() - t0 < 2 and checks
        # an error posted by a peer ends the wait at the next check
        def boom():
            raise RuntimeError("peer error")
        with pytest.raises(RuntimeError, match="peer error"):
            b.wait([b.pulled_slot(4)], 1, 10.0, boom, "pulled")
        assert digest_word("") == 0 and word_digest(0) == ""
        assert word_digest(digest_word("ffffffffffffffff")) == "ffffffffffffffff"
    finally:
        b.close()
