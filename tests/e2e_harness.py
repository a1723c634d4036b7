"""Multi-process end-to-end harness: one rollout process (FastAPI + controller + receiver
worker) and N trainer processes (torch.distributed gloo group), all through the public API.
Used by the CPU (gloo transport) and GPU (CUDA IPC, colocated on one GPU) tests."""
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


def _share_cores(nprocs: int) -> None:
    """Several processes on one host: split the cores between their intra-op thread pools
    (oversubscribed OpenMP teams spin against each other and slow every host op a hundredfold)."""
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // max(1, nprocs)))


def rollout_proc(port, q, n_syncs, model, mode, device, rlayout, dtype, late=False, direction=None,
                 exit_after=None, cfg_extra=None, nprocs=3, subset_prefix=None):
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    try:
        _share_cores(nprocs)
        if device != "cpu":
            torch.cuda.set_device(torch.device(device))
        app = FastAPI()
        ctl = WeightReceiverController(app, worker_num=1, timeout_s=60)
        lay = SGLangLayout(get_arch(model), **rlayout)
        params = lay.allocate(device=device, dtype=dtype)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60, **(cfg_extra or {}))
        # late: the reference's flow, tensors handed over at request_update
        recv = WeightReceiver(ctl.ipc_name, 0, meta, state_dict=None if late else views, config=cfg)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        q.put(("serving", None, None))
        results = []
        for i in range(n_syncs):
            if exit_after is not None and i == exit_after:
                q.put(("rollout-exit", i, None))
                q.close()
                q.join_thread()       # os._exit skips the queue's feeder thread: flush it first
                os._exit(0)           # leave between syncs: nothing of ours is in flight
            ok = recv.request_update(views if late else None, timeout=60)
            exp = lay.allocate(device=device, dtype=dtype, fill=True, seed=i)
            if subset_prefix is not None and i % 2:      # a partial sync: other entries keep seed i - 1
                prev = lay.allocate(device=device, dtype=dtype, fill=True, seed=i - 1)
                _m, ev = lay.to_wb(exp)
                _m, pv = lay.to_wb(prev)
                as_list = lambda v: v if isinstance(v, list) else [v]      # noqa: E731
                same = all(torch.equal(a.view(torch.uint8), b.view(torch.uint8))
                           for n in views
                           for a, b in zip(as_list(views[n]), as_list((ev if n.startswith(subset_prefix) else pv)[n])))
            else:
                same = all(torch.equal(params[n].view(torch.uint8) if params[n].dtype == torch.float8_e4m3fn else params[n],
                                       exp[n].view(torch.uint8) if exp[n].dtype == torch.float8_e4m3fn else exp[n])
                           for n in params)
            results.append(bool(ok) and same)
        stats = ctl.get_stats()
        q.put(("rollout", results, stats[0]["epoch"]))
        recv.stop()
        server.should_exit = True
        ctl.close()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc(), None))


def trainer_proc(rank, world, tport, url, q, n_syncs, model, mode, device, layouts, dtype, direction=None,
                 cfg_extra=None, trainer="megatron", subset_prefix=None):
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    try:
        _share_cores(world + 1)
        if device != "cpu":
            torch.cuda.set_device(torch.device(device))
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=world)
        if trainer == "fsdp":
            from weightbridge_b200.parallel.fsdp import FSDPLayout
            lay = FSDPLayout(get_arch(model), **layouts[rank])
        else:
            lay = MegatronLayout(get_arch(model), **layouts[rank])
        params = lay.allocate(device=device, dtype=dtype, seed=0)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60,
                             **({"direction": direction} if direction else {}), **(cfg_extra or {}))
        sender = WeightSender(mode, [url], config=cfg)
        sender.connect(meta)
        try:
            for i in range(n_syncs):
                if i:
                    lay.fill(params, seed=i)
                partial = subset_prefix is not None and i % 2
                sender.send(views, names=[n for n in views if n.startswith(subset_prefix)] if partial else None)
            q.put(("trainer", rank, sender.epoch))
        finally:
            sender.disconnect()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc(), rank))


def run(model, mode, trainer_layouts, rollout_layout, device="cpu", dtype=torch.float32, n_syncs=3, timeout=240,
        trainer_devices=None, late=False, direction=None, cfg_extra=None, trainer="megatron", subset_prefix=None):
    """``subset_prefix``: odd syncs send only the HF entries with that prefix (partial syncs)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hport, tport = _port(), _port()
    url = f"http://127.0.0.1:{hport}"
    world = len(trainer_layouts)
    procs = [ctx.Process(target=rollout_proc, args=(hport, q, n_syncs, model, mode, device, rollout_layout, dtype,
                                                    late, direction, None, cfg_extra, world + 1, subset_prefix))]
    tdev = trainer_devices or [device] * world
    procs += [ctx.Process(target=trainer_proc, args=(r, world, tport, url, q, n_syncs, model, mode, tdev[r],
                                                      trainer_layouts, dtype, direction, cfg_extra, trainer,
                                                      subset_prefix))
              for r in range(world)]
    procs[0].start()
    deadline = time.time() + timeout
    first = q.get(timeout=120)
    if first[0] == "error":
        procs[0].join(timeout=10)
        raise AssertionError(first[1])
    for p in procs[1:]:
        p.start()
    got = []
    try:
        while len(got) < world + 1 and time.time() < deadline:
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
            p.join(timeout=15)
            if p.is_alive():
                p.kill()
    roll = [g for g in got if g[0] == "rollout"]
    assert roll, f"no rollout result: {got}"
    assert roll[0][1] == [True] * n_syncs, roll
    assert roll[0][2] == n_syncs
    assert sorted(g[1] for g in got if g[0] == "trainer") == list(range(world))
    return got


# ------------------------------------------------------------------------------------------
# fan-out: one rollout process per replica (each its own engine), every trainer sends to all
# ------------------------------------------------------------------------------------------
def fanout_rollout_proc(port, q, n_syncs, model, mode, device, rlayout, dtype, nprocs):
    """One replica engine.  In mode "nvls" its parameters live in a VmmPool so that the pool
    can back a multicast object; ``recv.stop()`` runs on every path, so the pool is unbound
    (after the senders unmapped the object) before this process exits."""
    import threading
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    recv = None
    try:
        _share_cores(nprocs)
        torch.cuda.set_device(torch.device(device))
        app = FastAPI()
        ctl = WeightReceiverController(app, worker_num=1, timeout_s=60)
        lay = SGLangLayout(get_arch(model), **rlayout)
        if mode == "nvls":
            from weightbridge_b200.parallel.vmm import VmmPool
            pool = VmmPool(lay.pool_bytes(dtype), torch.device(device))
            params = lay.allocate(device=device, dtype=dtype, buffer=pool.params_buffer())
        else:
            params = lay.allocate(device=device, dtype=dtype, pool=True)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60)
        recv = WeightReceiver(ctl.ipc_name, 0, meta, state_dict=views, config=cfg)
        server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=server.run, daemon=True).start()
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        q.put(("serving", port, None))
        results = []
        for i in range(n_syncs):
            ok = recv.request_update(timeout=60)
            exp = lay.allocate(device=device, dtype=dtype, fill=True, seed=i)
            same = all(torch.equal(params[n].view(torch.uint8), exp[n].view(torch.uint8)) for n in params)
            results.append(bool(ok) and same)
            del exp
        q.put(("rollout", results, ctl.get_stats()[0]["epoch"]))
        server.should_exit = True
        ctl.close()
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc(), None))
    finally:
        if recv is not None:
            recv.stop()


def fanout_trainer_proc(rank, world, tport, urls, q, n_syncs, model, mode, device, layouts, dtype):
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.core.plan import OP_COPY_MC
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    sender = None
    try:
        _share_cores(world + len(urls))
        torch.cuda.set_device(torch.device(device))
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=rank, world_size=world)
        lay = MegatronLayout(get_arch(model), **layouts[rank])
        params = lay.allocate(device=device, dtype=dtype, seed=0)
        meta, views = lay.to_wb(params)
        cfg = TransferConfig(mode=mode, connect_timeout_s=60, sync_timeout_s=60)
        sender = WeightSender(mode, urls, config=cfg)
        sender.connect(meta)
        for i in range(n_syncs):
            if i:
                lay.fill(params, seed=i)
            sender.send(views)
        prog = sender.program
        mc_items = int(((prog.tables.items["op"] & 0xFF) == OP_COPY_MC).sum()) if prog is not None else 0
        q.put(("trainer", rank, {"epoch": sender.epoch, "mc_groups": len(sender._mc), "mc_items": mc_items,
                                 "targets": sorted(sender.targets)}))
    except Exception:
        import traceback
        q.put(("error", traceback.format_exc(), rank))
    finally:
        if sender is not None:
            sender.disconnect()
        if dist.is_initialized():
            dist.destroy_process_group()


def run_fanout(model, mode, trainer_layouts, rollout_layout, trainer_devices, replica_devices,
               dtype=torch.bfloat16, n_syncs=2, timeout=300):
    """Trainer ranks on ``trainer_devices`` sync into one replica engine per entry of
    ``replica_devices`` (identical layouts: a replica group).  Returns the trainers' reports
    (epoch, multicast groups, multicast work items).  Processes are given time to finish their
    teardown before anything is killed."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = len(trainer_layouts)
    nprocs = world + len(replica_devices)
    hports = [_port() for _ in replica_devices]
    tport = _port()
    rolls = [ctx.Process(target=fanout_rollout_proc, args=(hp, q, n_syncs, model, mode, dev, rollout_layout, dtype,
                                                            nprocs))
             for hp, dev in zip(hports, replica_devices)]
    for p in rolls:
        p.start()
    serving = 0
    while serving < len(rolls):
        item = q.get(timeout=120)
        if item[0] == "error":
            for p in rolls:
                p.join(timeout=120)
            raise AssertionError(item[1])
        serving += item[0] == "serving"
    urls = [f"http://127.0.0.1:{hp}" for hp in hports]
    trs = [ctx.Process(target=fanout_trainer_proc, args=(r, world, tport, urls, q, n_syncs, model, mode,
                                                          trainer_devices[r], trainer_layouts, dtype))
           for r in range(world)]
    for p in trs:
        p.start()
    got, errors = [], []
    deadline = time.time() + timeout
    try:
        while len(got) + len(errors) < nprocs and time.time() < deadline:
            try:
                item = q.get(timeout=1)
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in rolls + trs):
                    break
                continue
            (errors if item[0] == "error" else got).append(item)
    finally:
        for p in trs + rolls:           # trainers unmap first; replicas unbind after them
            p.join(timeout=180)
        for p in trs + rolls:
            if p.is_alive():
                p.kill()
    assert not errors, errors[0][1]
    roll = [g for g in got if g[0] == "rollout"]
    assert len(roll) == len(replica_devices), got
    for r in roll:
        assert r[1] == [True] * n_syncs, roll
        assert r[2] == n_syncs
    reports = {g[1]: g[2] for g in got if g[0] == "trainer"}
    assert sorted(reports) == list(range(world))
    return reports
