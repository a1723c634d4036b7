"""End-to-end control plane on CPU: FastAPI controller + ZMQ worker + TCPStore session + gloo.

The plumbing configuration: a tiny Llama-style decoder (2 layers, hidden 256, 4 heads of
dim 64, 2 KV heads, FFN 688, vocab 1024), fp32 N(0, 0.02) weights; Megatron TP=2 senders
(two processes) and one SGLang TP=1 receiver process, world size 3.  The receiver must match
the expected weights bit for bit after each of several syncs (new weights every sync).
"""
import torch

from tests.e2e_harness import run


def test_tiny_llama_tp2_to_tp1_gloo_world3():
    run("tiny-llama", "cpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1))


def test_tiny_qwen3_moe_ep2_to_tp1_fp8_gloo():
    """fp8 block quantisation on the sender side of the gloo path."""
    run("tiny-qwen3-moe", "cpu_direct", [dict(ep=2, ep_rank=0), dict(ep=2, ep_rank=1)],
        dict(tp=1, quant="fp8_experts"), dtype=torch.bfloat16, n_syncs=2)


def test_megatron_tp2_to_fp8_linear_gloo():
    """fp8 on every linear layer from Megatron's grouped QKV: 64-row KV groups are half a
    block, so each K/V block is shared by the two TP ranks, which exchange its amax."""
    run("tiny-qwen2-moe", "cpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)],
        dict(tp=1, quant="fp8_linear"), dtype=torch.bfloat16, n_syncs=2)


def test_redundant_expert_slots_fp8_gloo():
    """A rollout worker with redundant expert slots (SGLang EPLB placement), fp8 experts."""
    run("tiny-qwen3-moe", "cpu_direct", [dict(ep=2, ep_rank=0), dict(ep=2, ep_rank=1)],
        dict(tp=1, quant="fp8_experts", expert_slots=[0, 5, 2, 5, 7, 1, 3, 6, 4]),
        dtype=torch.bfloat16, n_syncs=2)


def test_deepseek_mla_tp2_ep2_to_tp1_fp8_experts_gloo():
    """DeepSeek-style model: MLA attention (the worker's derived w_kc / w_vc written with
    kv_b_proj), dense first layer, shared experts, router bias, fp8 routed experts; four
    Megatron ranks (TP 2 x EP 2) into one SGLang worker over the wire path."""
    run("tiny-deepseek-v3", "cpu_direct", [dict(tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)],
        dict(tp=1, quant="fp8_experts"), dtype=torch.bfloat16, n_syncs=2)


def test_deepseek_mla_gpu_direct_protocol_on_host():
    """The same model through the gpu_direct protocol in one process (work tables run by the
    C++ executor, host addresses): one op per destination shard, so w_kc / w_vc are written
    with their transposed strides straight from the trainer's kv up projection."""
    import threading
    from weightbridge_b200 import WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from tests.test_failures_cpu import Rollout, _cfg
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg, model="tiny-deepseek-v3", layout=dict(tp=1))
    try:
        lay = MegatronLayout(get_arch("tiny-deepseek-v3"), tp=1)
        params = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(params)
        with WeightSender("gpu_direct", [ro.url], config=cfg) as s:
            s.connect(meta)
            for seed in (3, 4):
                lay.fill(params, seed=seed)
                th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
                th.start()
                s.send(views)
                th.join(20)
                exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=seed)
                assert all(torch.equal(ro.params[n], exp[n]) for n in exp), seed
    finally:
        ro.close()


def test_glm4_moe_tp2_ep2_to_tp2_fp8_experts_gloo():
    """GLM-4.5 style (GQA with q/k/v bias, dense first layer, ungated shared experts, router
    bias): Megatron TP 2 x EP 2 into an SGLang worker with fp8 experts."""
    run("tiny-glm4-moe", "cpu_direct", [dict(tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)],
        dict(tp=1, quant="fp8_experts"), dtype=torch.bfloat16, n_syncs=2)


def test_deepseek_fused_shared_expert_slot_fp8_gloo():
    """The shared expert kept as a fifth slot of each layer's fp8 FusedMoE tensors: the two
    Megatron TP ranks each hold half of its rows, so its fp8 blocks are split between them
    (amax exchanged) and land in the fused slot."""
    slots = [[]] + [[0, 1, 2, 3, 4, 5, 6, 7, -1]] * 2
    run("tiny-deepseek-v3", "cpu_direct", [dict(tp=2, tp_rank=i) for i in range(2)],
        dict(tp=1, quant="fp8_experts", expert_slots=slots), dtype=torch.bfloat16, n_syncs=2)


def test_partial_syncs_with_split_fp8_blocks_gloo():
    """Odd syncs send layer 1 only: over the wire path, with K/V fp8 blocks split between the
    two TP ranks (amax exchanged within the partial sync); the rest keeps the previous sync's
    weights."""
    run("tiny-qwen2-moe", "cpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)],
        dict(tp=1, quant="fp8_linear"), dtype=torch.bfloat16, n_syncs=3, subset_prefix="model.layers.1.",
        cfg_extra=dict(wire_chunk_bytes=64 << 10))
