"""Public API across GPUs over NVLink: trainer processes on some GPUs, the rollout process on
another; the transfer kernel stores into the peer GPU's parameters through CUDA IPC."""
import pytest
import torch

from tests.e2e_harness import run

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def test_two_gpus_tiny_llama_tp1_to_tp1():
    _need(2)
    run("tiny-llama", "gpu_direct", [dict(tp=1)], dict(tp=1), device="cuda:1", dtype=torch.bfloat16,
        trainer_devices=["cuda:0"])


def test_two_gpus_fp8_experts_over_nvlink():
    _need(2)
    run("tiny-qwen3-moe", "gpu_direct", [dict(ep=1)], dict(tp=1, quant="fp8_experts"), device="cuda:1",
        dtype=torch.bfloat16, trainer_devices=["cuda:0"], n_syncs=2)


def test_three_gpus_two_senders_one_receiver():
    _need(3)
    run("tiny-qwen2", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1), device="cuda:2",
        dtype=torch.bfloat16, trainer_devices=["cuda:0", "cuda:1"])


def test_two_gpus_nccl_wire_mode():
    """Cross-node capable path: pack kernel -> NCCL send/recv -> unpack kernel."""
    _need(2)
    run("tiny-qwen2", "nccl", [dict(tp=1)], dict(tp=1), device="cuda:1", dtype=torch.bfloat16,
        trainer_devices=["cuda:0"])
