"""Failure detection across processes (no GPU): a trainer rank that dies after connect.

The surviving sender completes its part; the rollout worker's update fails with a clear
error long before its 30 s deadline (gloo reports the closed connection of the dead rank).
Failures are made on the host only: the rank's process exits between two calls.
"""
import multiprocessing as mp
import os
import queue
import socket
import time

import torch


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _trainer(rank, tport, url, q):
    torch.set_num_threads(2)            # three processes share the host's cores
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=2)
    lay = MegatronLayout(get_arch("tiny-llama"), tp=2, tp_rank=rank)
    p = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(p)
    cfg = TransferConfig(mode="cpu_direct", connect_timeout_s=30, sync_timeout_s=30)
    s = WeightSender("cpu_direct", [url], config=cfg)
    s.connect(meta)
    if rank == 1:
        time.sleep(1.0)
        os._exit(3)                      # dies between calls: nothing of it is in flight
    try:
        s.send(views)
        q.put(("trainer0", "ok"))
    except Exception as e:
        q.put(("trainer0", f"{type(e).__name__}: {e}"))
    time.sleep(15)                       # keep the session store (hosted here) up for the rollout


def _rollout(port, q):
    torch.set_num_threads(2)
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.control.receiver import ReceiveError
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    app = FastAPI()
    ctl = WeightReceiverController(app, worker_num=1, timeout_s=30)
    lay = SGLangLayout(get_arch("tiny-llama"), tp=1)
    p = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(p)
    recv = WeightReceiver(ctl.ipc_name, 0, meta, state_dict=views,
                          config=TransferConfig(mode="cpu_direct", sync_timeout_s=30))
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    threading.Thread(target=srv.run, daemon=True).start()
    while not srv.started:
        time.sleep(0.05)
    q.put(("serving", None))
    try:
        ok = recv.request_update(timeout=30)
        q.put(("rollout", f"returned {ok}"))
    except ReceiveError as e:
        q.put(("rollout", f"ReceiveError: {e}"))
    time.sleep(1)                        # let the queue's feeder flush before the process ends
    recv.stop()
    ctl.close()


def test_sender_rank_dying_after_connect_fails_the_update_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hport, tport = _port(), _port()
    roll = ctx.Process(target=_rollout, args=(hport, q))
    roll.start()
    assert q.get(timeout=120)[0] == "serving"
    trainers = [ctx.Process(target=_trainer, args=(r, tport, f"http://127.0.0.1:{hport}", q)) for r in range(2)]
    t0 = time.time()
    for t in trainers:
        t.start()
    got = {}
    try:
        while len(got) < 2:
            k, v = q.get(timeout=60)
            got[k] = (v, time.time() - t0)
    except queue.Empty:
        pass
    finally:
        for p in trainers + [roll]:
            p.join(timeout=20)
            if p.is_alive():
                p.kill()
    assert got.get("trainer0", ("",))[0] == "ok", got
    msg, dt = got["rollout"]
    assert msg.startswith("ReceiveError") and "closed" in msg.lower(), msg
    assert dt < 25, got                  # well inside the 30 s sync deadline


def _lagging_trainer(rank, tport, url, q, syncs):
    torch.set_num_threads(2)
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=2)
        lay = MegatronLayout(get_arch("tiny-llama"), tp=2, tp_rank=rank)
        p = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(p)
        cfg = TransferConfig(mode="cpu_direct", connect_timeout_s=30, sync_timeout_s=30)
        s = WeightSender("cpu_direct", [url], config=cfg)
        s.connect(meta)
        for i in range(syncs):
            if rank == 1 and i == syncs - 1:
                time.sleep(3.0)          # rank 0 finishes its last sync and leaves meanwhile
            s.send(views)
        s.disconnect()
        q.put((f"trainer{rank}", "ok"))
    except Exception as e:
        q.put((f"trainer{rank}", f"{type(e).__name__}: {e}"))


def _rollout_n(port, q, syncs):
    torch.set_num_threads(2)
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    app = FastAPI()
    ctl = WeightReceiverController(app, worker_num=1, timeout_s=30)
    lay = SGLangLayout(get_arch("tiny-llama"), tp=1)
    p = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(p)
    recv = WeightReceiver(ctl.ipc_name, 0, meta, state_dict=views,
                          config=TransferConfig(mode="cpu_direct", sync_timeout_s=30))
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    threading.Thread(target=srv.run, daemon=True).start()
    while not srv.started:
        time.sleep(0.05)
    q.put(("serving", None))
    try:
        oks = [recv.request_update(timeout=30) for _ in range(syncs)]
        exp = lay.allocate(dtype=torch.float32, fill=True)
        q.put(("rollout", "ok" if all(oks) and all(torch.equal(p[n], exp[n]) for n in p) else f"bad {oks}"))
    except Exception as e:
        q.put(("rollout", f"{type(e).__name__}: {e}"))
    time.sleep(1)
    recv.stop()
    ctl.close()


def test_rank0_leaving_first_keeps_the_session_for_a_lagging_rank():
    """Rank 0 hosts the session store.  It finishes its last sync and disconnects while rank 1
    is still 3 s away from its own last send: rank 0's disconnect keeps the store up until rank 1
    has left, so rank 1's last sync and the worker's update both complete."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hport, tport = _port(), _port()
    roll = ctx.Process(target=_rollout_n, args=(hport, q, 2))
    roll.start()
    assert q.get(timeout=120)[0] == "serving"
    trainers = [ctx.Process(target=_lagging_trainer, args=(r, tport, f"http://127.0.0.1:{hport}", q, 2))
                for r in range(2)]
    for t in trainers:
        t.start()
    got = {}
    try:
        while len(got) < 3:
            k, v = q.get(timeout=90)
            got[k] = v
    except queue.Empty:
        pass
    finally:
        for p in trainers + [roll]:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert got == {"trainer0": "ok", "trainer1": "ok", "rollout": "ok"}, got
