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
