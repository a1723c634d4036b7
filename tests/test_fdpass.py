"""File-descriptor passing between processes (used to share VMM pools and multicast objects)."""
import multiprocessing as mp
import os
import tempfile

from weightbridge_b200.parallel.fdpass import FdServer, fetch_fd


def _child(address, q):
    try:
        fd = fetch_fd(address, "pool")
        os.lseek(fd, 0, os.SEEK_SET)
        q.put(os.read(fd, 5))
        os.close(fd)
        try:
            fetch_fd(address, "missing")
            q.put("no error")
        except KeyError:
            q.put("missing ok")
    except Exception as e:
        q.put(repr(e))


def test_fd_roundtrip_between_processes():
    with tempfile.TemporaryFile() as f:
        f.write(b"hello")
        f.flush()
        srv = FdServer()
        srv.publish("pool", f.fileno())
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        p = ctx.Process(target=_child, args=(srv.address, q))
        p.start()
        assert q.get(timeout=30) == b"hello"
        assert q.get(timeout=30) == "missing ok"
        p.join(10)
        srv.close()
