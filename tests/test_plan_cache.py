"""Plans keyed by layout, not by address: the sender's relative binding and the on-disk
plan cache (a restarted trainer reuses the ops of its last run)."""
import json
import os
import threading

import numpy as np
import torch

from weightbridge_b200 import WeightSender
from weightbridge_b200.core.binding import bind
from weightbridge_b200.core.plan import lower_ops, phys_binding, plan_pair
from weightbridge_b200.core.plancache import PlanCache, plan_key, relative_binding
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout
from tests.test_failures_cpu import Rollout, _cfg, _sender


def _tables_equal(a, b):
    return all(np.array_equal(getattr(a, f), getattr(b, f)) for f in ("items", "qdescs", "qwork", "pieces")) \
        and a.piece_keys == b.piece_keys


def test_relative_binding_is_address_free_and_lowers_like_the_absolute_one():
    arch = get_arch("tiny-qwen3-moe")
    lay = MegatronLayout(arch, etp=4, etp_rank=1)
    p1, p2 = lay.allocate(dtype=torch.float32, fill=False), lay.allocate(dtype=torch.float32, fill=False)
    b1, b2 = bind(*lay.to_wb(p1)), bind(*lay.to_wb(p2))
    (r1, ptrs1), (r2, _ptrs2) = relative_binding(b1), relative_binding(b2)
    assert r1.to_json() == r2.to_json()
    rl = SGLangLayout(arch, tp=1, quant="fp8_experts")
    dst = phys_binding(bind(*rl.to_wb(rl.allocate(dtype=torch.float32, fill=False))))
    rel = lower_ops(plan_pair(r1, dst), ptrs1.__getitem__, lambda a: 0, receiver=3)
    ab = lower_ops(plan_pair(phys_binding(b1), dst), lambda a: 0, lambda a: 0, receiver=3)
    assert len(rel.pieces) and len(rel.items) and _tables_equal(rel, ab)


def test_plan_cache_round_trip_and_corrupt_entries(tmp_path):
    arch = get_arch("tiny-qwen3-moe")
    src, _ptrs = relative_binding(bind(*MegatronLayout(arch, etp=4, etp_rank=2).to_wb(
        MegatronLayout(arch, etp=4, etp_rank=2).allocate(dtype=torch.bfloat16, fill=False))))
    rl = SGLangLayout(arch, tp=1, quant="fp8_experts")
    dst = phys_binding(bind(*rl.to_wb(rl.allocate(dtype=torch.bfloat16, fill=False))))
    whole, _p = relative_binding(bind(*MegatronLayout(arch, tp=1).to_wb(
        MegatronLayout(arch, tp=1).allocate(dtype=torch.bfloat16, fill=False))))
    ops = plan_pair(src, dst) + plan_pair(whole, dst)      # split pieces and whole blocks
    key = plan_key(src.to_json(), dst.to_json(), None)
    assert key != plan_key(src.to_json(), dst.to_json(), ["model.norm.weight"])
    cache = PlanCache(str(tmp_path / "plans"))
    assert cache.get(key) is None and cache.misses == 1
    cache.put(key, ops)
    back = cache.get(key)
    assert back == ops and cache.hits == 1
    assert {o.kind for o in back} >= {"copy", "quant", "squant"}
    base = lambda a: 4096 * (a + 1)                     # noqa: E731
    assert _tables_equal(lower_ops(back, base, base), lower_ops(ops, base, base))
    path = tmp_path / "plans" / f"{key}.json"
    path.write_text(path.read_text()[:100])                 # a torn or foreign file is a miss
    assert cache.get(key) is None
    path.write_text(json.dumps({"format": 1, "key": "other", "ops": []}))
    assert cache.get(key) is None
    assert not [f for f in os.listdir(tmp_path / "plans") if f.endswith(".tmp")]


def test_restarted_sender_reuses_its_plans_from_disk(tmp_path):
    """A second sender (as after a trainer restart: new tensors, same layout) plans nothing:
    its ops come from the cache directory, and the sync is still exact."""
    cfg = _cfg(mode="gpu_direct", plan_cache_dir=str(tmp_path))
    ro = Rollout(cfg)
    try:
        for run, seed in enumerate((0, 5)):
            lay, params, meta, views = _sender(cfg)
            lay.fill(params, seed=seed)
            s = WeightSender("gpu_direct", [ro.url], config=cfg)
            s.connect(meta)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(views)
            th.join(20)
            assert (s._plan_cache.hits, s._plan_cache.misses) == ((0, 1) if run == 0 else (1, 0))
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=seed)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), run
            s.disconnect()
        assert len([f for f in os.listdir(tmp_path) if f.endswith(".json")]) == 1
    finally:
        ro.close()
