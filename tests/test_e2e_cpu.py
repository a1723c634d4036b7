"""End-to-end control plane on CPU: FastAPI controller + ZMQ worker + TCPStore session + gloo.

The plumbing configuration: a tiny Llama-style decoder (2 layers, hidden 256, 4 heads of
dim 64, 2 KV heads, FFN 688, vocab 1024), fp32 N(0, 0.02) weights; Megatron TP=2 senders
(two processes) and one SGLang TP=1 receiver process, world size 3.  The receiver must match
the expected weights bit for bit after each of several syncs (new weights every sync).
"""
import multiprocessing as mp
import os
import queue
import socket
import time

import pytest
import torch




def _rollout(port, q, n_syncs, model, mode):
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    try:
        app = FastAPI()
        ctl = WeightReceiverController(app, worker_num=1, timeout_s=30)
        lay = SGLangLayout(get_arch(model), tp=1)
        params = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60)
        recv = WeightReceiver(ctl.ipc_name, 0, meta, state_dict=views, config=cfg)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        th = threading.Thread(target=server.run, daemon=True)
        th.start()
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        results = []
        for i in range(n_syncs):
            ok = recv.request_update(timeout=60)
            exp = lay.allocate(dtype=torch.float32, fill=True, seed=i)
            results.append(bool(ok) and all(torch.equal(params[n], exp[n]) for n in params))
        stats = ctl.get_stats()
        q.put(("rollout", results, stats[0]["epoch"]))
        recv.stop()
        server.should_exit = True
        ctl.close()
    except Exception as e:  # report instead of hanging the parent
        import traceback
        q.put(("error", traceback.format_exc(), None))


def _trainer(rank, tport, url, q, n_syncs, model, mode):
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=2)
        lay = MegatronLayout(get_arch(model), tp=2, tp_rank=rank)
        params = lay.allocate(dtype=torch.float32, seed=0)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60)
        sender = WeightSender(mode, [url], config=cfg)
        sender.connect(meta)
        for i in range(n_syncs):
            if i:
                lay.fill(params, seed=i)
            sender.send(views)
        q.put(("trainer", rank, sender.epoch))
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc(), rank))


def _run(model, mode, n_syncs=3, timeout=180):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hport, tport = _port(), _port()
    url = f"http://127.0.0.1:{hport}"
    procs = [ctx.Process(target=_rollout, args=(hport, q, n_syncs, model, mode))]
    procs += [ctx.Process(target=_trainer, args=(r, tport, url, q, n_syncs, model, mode)) for r in range(2)]
    for p in procs:
        p.start()
    got = []
    deadline = time.time() + timeout
    try:
        while len(got) < 3 and time.time() < deadline:
            try:
                item = q.get(timeout=1)
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
                continue
            if item[0] == "error":
                raise AssertionError(item[1])
            got.append(item)
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return got


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["cpu_direct"])
def test_tiny_llama_tp2_to_tp1_gloo_world3(mode):
    got = _run("tiny-llama", mode)
    roll = [g for g in got if g[0] == "rollout"]
    assert roll, got
    assert roll[0][1] == [True, True, True]
    assert roll[0][2] == 3
    assert sorted(g[1] for g in got if g[0] == "trainer") == [0, 1]
