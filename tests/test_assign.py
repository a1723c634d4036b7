"""Source assignment: replica groups, overlap rules and load balancing."""
import pytest
import torch

from weightbridge_b200 import WeightData
from weightbridge_b200.control.assign import assign_sources, expected_senders, replica_groups
from weightbridge_b200.core.shard import box_copy
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout


def _meta(lay, param_specs):
    params = {n: torch.empty(s, dtype=torch.bfloat16, device="meta") for n, s in param_specs.items()}
    return lay.to_wb(params)[0]


def _bytes(plan, smetas, rmetas):
    out = {}
    for s, rs in plan.items():
        n = 0
        for r, names in rs.items():
            for name in names:
                for a in smetas[s].shards(name):
                    for b in rmetas[r].shards(name):
                        bc = box_copy(a, b)
                        if bc is not None:
                            n += bc.numel * 2
        out[s] = n
    return out


def test_ep4_to_tp4_dense_weights_spread_over_senders():
    arch = get_arch("qwen3-30b-a3b").with_(num_layers=4)
    smetas = []
    for r in range(4):
        lay = MegatronLayout(arch, ep=4, ep_rank=r)
        smetas.append(_meta(lay, lay.param_shapes()))
    rmetas = {}
    for r in range(4):
        lay = SGLangLayout(arch, tp=4, tp_rank=r, moe_ep=4)
        rmetas[4 + r] = _meta(lay, {n: s for n, (s, _k) in lay.param_specs().items()})
    plan = assign_sources(smetas, rmetas)
    loads = _bytes(plan, smetas, rmetas)
    assert len(loads) == 4
    assert max(loads.values()) / min(loads.values()) < 1.05, loads
    # experts come only from their EP owner
    for s, rs in plan.items():
        for r, names in rs.items():
            for n in names:
                if ".experts." in n:
                    e = int(n.split(".experts.")[1].split(".")[0])
                    assert e // 32 == s
    # lowest-rank-wins is available for comparison
    low = assign_sources(smetas, rmetas, load_balance=False)
    assert max(_bytes(low, smetas, rmetas).values()) > max(loads.values())


def test_partial_overlap_between_senders_raises():
    a = WeightData({"w": {"shard": [(0, 3, 4), (0, 4, 4)], "dtype": "float32"}})
    b = WeightData({"w": {"shard": [(2, 4, 4), (0, 4, 4)], "dtype": "float32"}})
    r = WeightData({"w": {"shard": [(0, 4, 4), (0, 4, 4)], "dtype": "float32"}})
    with pytest.raises(ValueError, match="Partial shard overlap"):
        assign_sources([a, b], {2: r})


def test_replicas_and_expected_senders():
    full = {"w": {"shard": [(0, 4, 4), (0, 4, 4)], "dtype": "float32"}}
    halves = [WeightData({"v": {"shard": [(0, 2, 4)], "dtype": "float32"}, **full}),
              WeightData({"v": {"shard": [(2, 4, 4)], "dtype": "float32"}, **full})]
    groups = replica_groups(halves)
    assert groups["w"] == [[0, 1]] and groups["v"] == [[0], [1]]
    recv = {2: WeightData({"w": full["w"], "v": {"shard": [(0, 4, 4)], "dtype": "float32"}}),
            3: WeightData({"w": full["w"]})}
    plan = assign_sources(halves, recv)
    # receiver 2 needs both halves of v: both senders; w goes to one of them each
    assert expected_senders(plan, 2) == [0, 1]
    w_senders = [s for s in plan for r in plan[s] for n in plan[s][r] if n == "w"]
    assert sorted(w_senders) == [0, 1]      # the two copies of w spread over the two replicas


def test_replica_consistent_assignment_serves_every_replica_alike():
    """Multicast fan-out (Llama TP2 x PP2 -> 4 TP1 replicas): with ``replica_consistent`` every
    sender writes the same entries to every replica (so one multicast store serves them all),
    each replica still receives every entry exactly once, and TP-replicated entries (layer
    norms) are still spread over the TP ranks.  Without it the per-replica balancing gives
    replicas different sources for those entries."""
    arch = get_arch("tiny-llama")
    smetas = []
    for pp in range(2):
        for tp in range(2):
            lay = MegatronLayout(arch, tp=2, pp=2, tp_rank=tp, pp_rank=pp)
            smetas.append(_meta(lay, lay.param_shapes()))
    rl = SGLangLayout(arch, tp=1)
    rmetas = {4 + j: _meta(rl, {n: sh for n, (sh, _k) in rl.param_specs().items()}) for j in range(4)}
    plan = assign_sources(smetas, rmetas, replica_consistent=True)
    for s, rs in plan.items():
        lists = [rs.get(r, []) for r in sorted(rmetas)]
        assert all(x == lists[0] for x in lists), s
    for r, meta in rmetas.items():
        got = sorted(n for s in plan for n in plan[s].get(r, []))
        # an entry split by TP arrives from both TP ranks of its stage, a replicated one from one
        assert set(got) == set(meta.names())
    norms = [n for n in rmetas[4].names() if "norm" in n]
    owners = {n: [s for s in plan if n in plan[s].get(4, [])] for n in norms}
    assert all(len(o) == 1 for o in owners.values())
    assert len({o[0] for o in owners.values()}) > 2          # spread over both TP ranks of both stages
    loose = assign_sources(smetas, rmetas)
    assert any(len({tuple(rs.get(r, [])) for r in rmetas}) > 1 for rs in loose.values())


def test_replicated_entries_come_from_the_receivers_own_gpu():
    """Trainer DP 2 (two identical TP1 ranks on GPUs A and B) into two colocated TP1 workers on
    A and B: each worker takes every entry from the rank on its own GPU (HBM copies), where the
    GPU-blind assignment balances bytes across both ranks (half of them over NVLink)."""
    arch = get_arch("tiny-llama")
    lay = MegatronLayout(arch, tp=1)
    smetas = [_meta(lay, lay.param_shapes()) for _ in range(2)]
    rl = SGLangLayout(arch, tp=1)
    rmetas = {2: _meta(rl, {n: sh for n, (sh, _k) in rl.param_specs().items()}),
              3: _meta(rl, {n: sh for n, (sh, _k) in rl.param_specs().items()})}
    plan = assign_sources(smetas, rmetas, sender_gpus=["A", "B"], receiver_gpus={2: "A", 3: "B"})
    assert set(plan) == {0, 1}
    assert set(plan[0]) == {2} and set(plan[1]) == {3}
    assert sorted(plan[0][2]) == sorted(rmetas[2].names()) and sorted(plan[1][3]) == sorted(rmetas[3].names())
    blind = assign_sources(smetas, rmetas)
    assert any(len(rs) > 1 for rs in blind.values())               # some entries cross GPUs
    # a worker on a GPU no trainer rank holds balances as before
    far = assign_sources(smetas, rmetas, sender_gpus=["A", "B"], receiver_gpus={2: "C", 3: "D"})
    assert _bytes(far, smetas, rmetas) == _bytes(blind, smetas, rmetas)
