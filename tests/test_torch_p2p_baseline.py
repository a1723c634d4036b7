"""The torch.distributed baseline (the reference's algorithm) on gloo, world size 3."""
import multiprocessing as mp
import socket

import torch


def _run(rank, port, q):
    import torch.distributed as dist
    from weightbridge_b200.baselines.torch_p2p import build_plan, sync
    from weightbridge_b200.core.binding import bind
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=3)
        arch = get_arch("tiny-llama")
        if rank < 2:
            lay = MegatronLayout(arch, tp=2, tp_rank=rank)
            params = lay.allocate(dtype=torch.float32)
        else:
            lay = SGLangLayout(arch, tp=1)
            params = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(params)
        plan = build_plan(rank, 3, meta, rank < 2, "cpu")
        sync(plan, bind(meta, views))
        ok = True
        if rank == 2:
            exp = lay.allocate(dtype=torch.float32, fill=True)
            ok = all(torch.equal(params[n], exp[n]) for n in params)
        q.put((rank, ok))
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


def test_torch_p2p_baseline_gloo():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_run, args=(r, port, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(3))
    for p in ps:
        p.join(30)
    assert res == {0: True, 1: True, 2: True}, res
