"""FSDP / DTensor trainer layout (parallel/fsdp.py): torch.chunk shard boxes, resharding into
SGLang layouts (bf16 and fp8 with blocks split across FSDP ranks), DTensor conversion."""
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from weightbridge_b200.core.binding import bind
from weightbridge_b200.core.plan import lower_ops, phys_binding, plan_pair
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.ops.executor import cpu_execute, cpu_piece_amax
from weightbridge_b200.parallel.fsdp import FSDPLayout, chunk_rows, shard_box
from weightbridge_b200.parallel.sglang import SGLangLayout

ABS = lambda _a: 0


def _u8(t):
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


@pytest.mark.parametrize("n", [1, 5, 7, 128, 171, 1000])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_chunk_rows_match_torch_chunk(n, world):
    parts = torch.arange(n).chunk(world)
    for r in range(world):
        l, h = chunk_rows(n, world, r)
        got = list(range(l, h))
        want = parts[r].tolist() if r < len(parts) else []
        assert got == want
        assert (shard_box((n, 4), world, r) is None) == (not want)


def _reshard(world, rollout, dtype):
    arch = get_arch("tiny-llama-fp8")
    senders = []
    for i in range(world):
        lay = FSDPLayout(arch, world=world, rank=i)
        p = lay.allocate(dtype=dtype)
        meta, views = lay.to_wb(p)
        senders.append((p, phys_binding(bind(meta, views))))
    out = []
    for rl in rollout:
        rp = rl.allocate(dtype=dtype)
        rmeta, rviews = rl.to_wb(rp)
        rphys = phys_binding(bind(rmeta, rviews))
        tables = [lower_ops(plan_pair(sphys, rphys), ABS, ABS, receiver=0) for _p, sphys in senders]
        block = {}
        for t in tables:
            for k, a in zip(t.piece_keys, cpu_piece_amax(t)):
                block[k] = max(block.get(k, 0.0), float(a))
        for t in tables:
            cpu_execute(t, np.array([block[k] for k in t.piece_keys], dtype=np.float32))
        out.append((rl, rp, sum(len(t.pieces) for t in tables)))
    return out


def test_fsdp_world3_to_sglang_tp2_bf16():
    arch = get_arch("tiny-llama-fp8")
    for rl, rp, _n in _reshard(3, [SGLangLayout(arch, tp=2, tp_rank=i) for i in range(2)], torch.bfloat16):
        exp = rl.allocate(dtype=torch.bfloat16, fill=True)
        assert all(torch.equal(rp[n], exp[n]) for n in rp)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fsdp_world3_to_sglang_fp8_linear_split_blocks(dtype):
    """171-row FSDP shards cut the 128-row blocks of every fp8 linear layer."""
    arch = get_arch("tiny-llama-fp8")
    (rl, rp, pieces), = _reshard(3, [SGLangLayout(arch, tp=1, quant="fp8_linear")], dtype)
    assert pieces > 0
    exp = rl.allocate(dtype=dtype, fill=True)
    for n in rp:
        assert torch.equal(_u8(rp[n]), _u8(exp[n])), n


def test_fsdp_to_fp8_rollout_over_gloo():
    """Three FSDP ranks, one fp8_linear rollout worker, through the public API."""
    from tests.e2e_harness import run
    run("tiny-llama-fp8", "cpu_direct", [dict(world=3, rank=i) for i in range(3)],
        dict(tp=1, quant="fp8_linear"), dtype=torch.bfloat16, n_syncs=2, trainer="fsdp")


def _dtensor_rank(rank, port, q):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor
    from weightbridge_b200.parallel.fsdp import convert_to_wb
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    mesh = init_device_mesh("cpu", (2,))
    w = torch.arange(20, dtype=torch.float32).view(5, 4)
    named = {"a.weight": distribute_tensor(w, mesh, [Shard(0)]),
             "b.weight": distribute_tensor(w.t().contiguous(), mesh, [Shard(1)]),
             "c.weight": distribute_tensor(w, mesh, [Replicate()]),
             "d.bias": torch.ones(3)}
    meta, views = convert_to_wb(named)
    q.put((rank, {n: meta.shards(n)[0] for n in meta.names()},
           {n: views[n].tolist() for n in views}))
    dist.destroy_process_group()


def test_dtensor_conversion_two_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dtensor_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict((r, (b, v)) for r, b, v in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(10)
    w = torch.arange(20, dtype=torch.float32).view(5, 4)
    b0, v0 = got[0]
    b1, v1 = got[1]
    assert b0["a.weight"] == [(0, 3, 5), (0, 4, 4)] and b1["a.weight"] == [(3, 5, 5), (0, 4, 4)]
    assert v0["a.weight"] == w[:3].tolist() and v1["a.weight"] == w[3:].tolist()
    assert b0["b.weight"] == [(0, 4, 4), (0, 3, 5)] and b1["b.weight"] == [(0, 4, 4), (3, 5, 5)]
    assert b0["c.weight"] == [(0, 5, 5), (0, 4, 4)] == b1["c.weight"]
    assert b0["d.bias"] == [(0, 3, 3)]


def _dtensor_2d_rank(rank, port, q):
    try:
        _dtensor_2d_body(rank, port, q)
    except Exception:
        import traceback
        q.put((rank, {"error": (None, traceback.format_exc())}))


def _dtensor_2d_body(rank, port, q):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor
    from weightbridge_b200.parallel.fsdp import convert_to_wb
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=4)
    mesh = init_device_mesh("cpu", (2, 2))
    w = torch.arange(7 * 6, dtype=torch.float32).view(7, 6)
    from torch.distributed.tensor.placement_types import _StridedShard
    w8 = torch.arange(8 * 6, dtype=torch.float32).view(8, 6)
    named = {"hsdp": distribute_tensor(w, mesh, [Replicate(), Shard(0)]),
             "two_dims": distribute_tensor(w, mesh, [Shard(0), Shard(1)]),
             "nested": distribute_tensor(w, mesh, [Shard(0), Shard(0)]),
             "fsdp_on_tp": distribute_tensor(w8, mesh, [_StridedShard(0, split_factor=2), Shard(0)])}
    meta, views = convert_to_wb(named)
    out = {}
    for n in meta.names():
        box = meta.shards(n)[0]
        ref = w8 if n == "fsdp_on_tp" else w
        out[n] = (box, torch.equal(views[n], ref[tuple(slice(l, r) for l, r, _ in box)]))
    q.put((rank, out))
    dist.destroy_process_group()


def test_dtensor_conversion_2d_mesh():
    """(Replicate, Shard(0)), (Shard(0), Shard(1)), nested (Shard(0), Shard(0)) and FSDP's
    (_StridedShard(0), Shard(0)) on a 2 x 2 mesh: every rank's box selects exactly its local
    tensor."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dtensor_2d_rank, args=(r, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(4))
    for p in ps:
        p.join(10)
    for r, out in got.items():
        assert "error" not in out, out.get("error")
        assert all(ok for _box, ok in out.values()), (r, out)
    # nested: rows 0-3 split 2-2 within the first mesh row, rows 4-6 split 2-1 in the second
    assert sorted(got[r]["nested"][0][0] for r in range(4)) == [(0, 2, 7), (2, 4, 7), (4, 6, 7), (6, 7, 7)]
    # FSDP (strided, mesh dim 0) on top of TP (mesh dim 1): TP halves first, then FSDP halves
    assert got[1]["fsdp_on_tp"][0][0] == (4, 6, 8) and got[2]["fsdp_on_tp"][0][0] == (2, 4, 8)


def test_hf_layout_receives_from_megatron():
    """A rollout holding the plain HF state_dict (HFLayout) from Megatron TP2 shards."""
    from weightbridge_b200 import HFLayout
    from weightbridge_b200.parallel.megatron import MegatronLayout
    arch = get_arch("tiny-qwen2")
    senders = []
    for i in range(2):
        lay = MegatronLayout(arch, tp=2, tp_rank=i)
        p = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(p)
        senders.append((p, phys_binding(bind(meta, views))))
    hl = HFLayout(arch)
    hp = hl.allocate(dtype=torch.float32, fill=False)
    hmeta, hviews = hl.to_wb(hp)
    rphys = phys_binding(bind(hmeta, hviews))
    for _p, sphys in senders:
        cpu_execute(lower_ops(plan_pair(sphys, rphys), ABS, ABS))
    exp = hl.allocate(dtype=torch.float32, fill=True)
    assert set(hp) == {n for n, _s in arch.hf_tensors()}
    assert all(torch.equal(hp[n], exp[n]) for n in exp)
