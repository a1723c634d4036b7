"""Config 5's control plane in miniature on CPU: eight Megatron TP8 trainer processes sync into
two rollout engines, each one process whose controller serves four TP4 workers (a worker
thread each), over gloo wires (``cpu_direct``).  Every worker of both engines must hold its
expected shard bit for bit after each sync; the source assignment, the session handshakes, the
per-engine controllers and the arm reach 16 receivers' worth of targets (8 workers x the senders
that overlap each).  The GPU layout of the same shape is ``bench.py --config llama70b-colocated``."""
import multiprocessing as mp
import queue
import time

import torch

from tests.e2e_harness import _port, _share_cores

MODEL = "tiny-llama-tp8"


def _engine(port, q, engine, tp, n_syncs, nprocs):
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    try:
        _share_cores(nprocs)
        app = FastAPI()
        ctl = WeightReceiverController(app, worker_num=tp, timeout_s=60)
        cfg = TransferConfig(mode="cpu_direct", connect_timeout_s=60, sync_timeout_s=60)
        lays = [SGLangLayout(get_arch(MODEL), tp=tp, tp_rank=i) for i in range(tp)]
        params = [lay.allocate(dtype=torch.float32) for lay in lays]
        recvs = []
        for i, (lay, p) in enumerate(zip(lays, params)):
            meta, views = lay.to_wb(p)
            recvs.append(WeightReceiver(ctl.ipc_name, i, meta, state_dict=views, config=cfg))
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        q.put(("serving", engine))
        results = []
        for s in range(n_syncs):
            oks = [None] * tp
            ths = [threading.Thread(target=lambda i=i: oks.__setitem__(i, recvs[i].request_update(timeout=60)))
                   for i in range(tp)]
            for t in ths:
                t.start()
            for t in ths:
                t.join(90)
            same = []
            for lay, p in zip(lays, params):
                exp = lay.allocate(dtype=torch.float32, fill=True, seed=s)
                same.append(all(torch.equal(p[n], exp[n]) for n in p))
            results.append(all(oks) and all(same))
        q.put(("engine", engine, results, [r.epoch for r in recvs]))
        for r in recvs:
            r.stop()
        server.should_exit = True
        ctl.close()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc()))


def _trainer(rank, world, tport, urls, q, n_syncs, nprocs):
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    try:
        _share_cores(nprocs)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=world)
        lay = MegatronLayout(get_arch(MODEL), tp=world, tp_rank=rank)
        params = lay.allocate(dtype=torch.float32, seed=0)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode="cpu_direct", connect_timeout_s=60, sync_timeout_s=60)
        sender = WeightSender("cpu_direct", urls, config=cfg)
        sender.connect(meta)
        try:
            for i in range(n_syncs):
                if i:
                    lay.fill(params, seed=i)
                sender.send(views)
            q.put(("trainer", rank, sender.epoch, len(sender.targets)))
        finally:
            sender.disconnect()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc()))


def test_tp8_trainer_into_two_tp4_engines_gloo():
    world, tp, engines, n_syncs = 8, 4, 2, 2
    nprocs = world + engines
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hports = [_port() for _ in range(engines)]
    tport = _port()
    eps = [ctx.Process(target=_engine, args=(hp, q, e, tp, n_syncs, nprocs)) for e, hp in enumerate(hports)]
    for p in eps:
        p.start()
    serving = 0
    while serving < engines:
        item = q.get(timeout=180)
        assert item[0] != "error", item[1]
        serving += 1
    urls = [f"http://127.0.0.1:{hp}" for hp in hports]
    tps = [ctx.Process(target=_trainer, args=(r, world, tport, urls, q, n_syncs, nprocs)) for r in range(world)]
    for p in tps:
        p.start()
    got = []
    deadline = time.time() + 300
    try:
        while len(got) < nprocs and time.time() < deadline:
            try:
                item = q.get(timeout=1)
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in eps + tps):
                    break
                continue
            assert item[0] != "error", item[1]
            got.append(item)
    finally:
        for p in tps + eps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    eng = sorted(g for g in got if g[0] == "engine")
    assert [g[1] for g in eng] == list(range(engines)), got
    for g in eng:
        assert g[2] == [True] * n_syncs and g[3] == [n_syncs] * tp, g
    tr = sorted(g for g in got if g[0] == "trainer")
    assert [g[1] for g in tr] == list(range(world)) and all(g[2] == n_syncs for g in tr)
    # a TP8 rank's rows land in one TP4 worker per engine, its replicated entries in any of them
    assert all(g[3] >= engines for g in tr)
