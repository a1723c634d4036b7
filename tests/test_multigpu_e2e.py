"""Public API across GPUs over NVLink: trainer processes on some GPUs, the rollout process on
another; the transfer kernel stores into the peer GPU's parameters through CUDA IPC."""
import pytest
import torch

from tests.e2e_harness import run

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


# not yet run on B200s: reported, but a failure does not stop the suite (pytest -x)
FIRST_RUN = pytest.mark.xfail(reason="first run on B200s pending", strict=False)


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


@FIRST_RUN
def test_three_gpus_two_senders_one_receiver():
    _need(3)
    run("tiny-qwen2", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1), device="cuda:2",
        dtype=torch.bfloat16, trainer_devices=["cuda:0", "cuda:1"])


@pytest.mark.parametrize("chunk", [0, pytest.param(64 << 10, marks=FIRST_RUN)])
def test_two_gpus_nccl_wire_mode(chunk):
    """Cross-node capable path: pack kernel -> NCCL send/recv -> unpack kernel, as one message
    per peer (chunk 0) or as many 64 KiB chunks through two buffers per peer."""
    _need(2)
    run("tiny-qwen2", "nccl", [dict(tp=1)], dict(tp=1), device="cuda:1", dtype=torch.bfloat16,
        trainer_devices=["cuda:0"], cfg_extra={"wire_chunk_bytes": chunk})


def _leaving_trainer(tport, url, q):
    import torch.distributed as dist
    from weightbridge_b200 import TransferConfig, WeightSender
    from weightbridge_b200.control.sender import TransferError
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{tport}", rank=0, world_size=1)
    lay = MegatronLayout(get_arch("tiny-llama"), tp=1)
    params = lay.allocate(device="cuda:0", dtype=torch.bfloat16)
    meta, views = lay.to_wb(params)
    cfg = TransferConfig(mode="gpu_direct", connect_timeout_s=60, sync_timeout_s=5, http_timeout_s=5)
    s = WeightSender("gpu_direct", [url], config=cfg)
    s.connect(meta)
    s.send(views)
    q.put(("first-sync", True, None))
    import time
    t0 = time.time()
    try:
        s.send(views)
        q.put(("second-sync", "no error", time.time() - t0))
    except (TransferError, Exception) as e:
        q.put(("second-sync", type(e).__name__, time.time() - t0))


@FIRST_RUN
def test_receiver_leaving_between_syncs_fails_the_next_send():
    """A rollout process exits between two syncs (nothing in flight); the trainer's next send
    reports an error within its deadline instead of hanging, and launches no kernel into the
    departed receiver's memory (the launch waits for the receiver's ready key)."""
    import multiprocessing as mp
    import os
    _need(2)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from tests.e2e_harness import _port, rollout_proc
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hport, tport = _port(), _port()
    roll = ctx.Process(target=rollout_proc, args=(hport, q, 2, "tiny-llama", "gpu_direct", "cuda:1", dict(tp=1),
                                                  torch.bfloat16, False, "push", 1))
    roll.start()
    assert q.get(timeout=120)[0] == "serving"
    tr = ctx.Process(target=_leaving_trainer, args=(tport, f"http://127.0.0.1:{hport}", q))
    tr.start()
    got = {}
    try:
        for _ in range(3):
            k, v, t = q.get(timeout=120)
            got[k] = (v, t)
    finally:
        for p in (tr, roll):
            p.join(30)
            if p.is_alive():
                p.kill()
    assert got["first-sync"][0] is True
    assert got["second-sync"][0] != "no error"
    assert got["second-sync"][1] < 30


@FIRST_RUN
def test_two_gpus_deepseek_mla_over_nvlink():
    """MLA (w_kc / w_vc written with kv_b_proj) and fp8 experts, trainer on GPU 0, worker on GPU 1."""
    _need(2)
    run("tiny-deepseek-v3", "gpu_direct", [dict(tp=1)], dict(tp=1, quant="fp8_experts"), device="cuda:1",
        dtype=torch.bfloat16, trainer_devices=["cuda:0"], n_syncs=2)
