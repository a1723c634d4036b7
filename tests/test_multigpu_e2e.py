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


@pytest.mark.parametrize("chunk", [0, 64 << 10])
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
        while "second-sync" not in got:      # "rollout-exit" may arrive in any order, or not at all
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


def test_two_gpus_deepseek_mla_over_nvlink():
    """MLA (w_kc / w_vc written with kv_b_proj) and fp8 experts, trainer on GPU 0, worker on GPU 1."""
    _need(2)
    run("tiny-deepseek-v3", "gpu_direct", [dict(tp=1)], dict(tp=1, quant="fp8_experts"), device="cuda:1",
        dtype=torch.bfloat16, trainer_devices=["cuda:0"], n_syncs=2)


# -- one-to-many fan-out: one engine per replica, identical layouts (a replica group) ---------
def test_unicast_fanout_one_sender_two_replicas():
    """The default fan-out: the sender's kernel stores every chunk once per replica."""
    _need(3)
    from tests.e2e_harness import run_fanout
    rep = run_fanout("tiny-llama", "gpu_direct", [dict(tp=1)], dict(tp=1), ["cuda:0"], ["cuda:1", "cuda:2"])
    assert rep[0]["mc_groups"] == 0 and rep[0]["mc_items"] == 0


def test_nvls_fanout_one_sender_two_replicas():
    """Mode "nvls": the two replicas' VMM pools and a scratch pool on the sender's GPU back one
    multicast object; the kernel's multimem stores reach both replicas in one write.  Both
    replicas verify bit for bit, and the sender's program holds multicast items."""
    _need(3)
    from tests.e2e_harness import run_fanout
    from weightbridge_b200.parallel.nvls import nvls_supported
    if not nvls_supported(0):
        pytest.skip("no NVLink multicast on this machine")
    rep = run_fanout("tiny-llama", "nvls", [dict(tp=1)], dict(tp=1), ["cuda:0"], ["cuda:1", "cuda:2"])
    assert rep[0]["mc_groups"] == 1 and rep[0]["mc_items"] > 0


def test_nvls_fanout_two_pipeline_stages_two_replicas():
    """Trainer PP 2 (each stage's sender writes its layers) into two TP1 replicas by multicast."""
    _need(4)
    from tests.e2e_harness import run_fanout
    from weightbridge_b200.parallel.nvls import nvls_supported
    if not nvls_supported(0):
        pytest.skip("no NVLink multicast on this machine")
    rep = run_fanout("tiny-llama", "nvls", [dict(tp=1, pp=2, pp_rank=0), dict(tp=1, pp=2, pp_rank=1)], dict(tp=1),
                     ["cuda:0", "cuda:1"], ["cuda:2", "cuda:3"])
    assert all(r["mc_groups"] == 1 and r["mc_items"] > 0 for r in rep.values())


def test_nvls_fanout_sender_on_a_replica_gpu():
    """Two GPUs: the sender shares GPU 0 with one replica (whose pool backs that device's share
    of the multicast object), the other replica is on GPU 1; both verify bit for bit."""
    _need(2)
    from tests.e2e_harness import run_fanout
    from weightbridge_b200.parallel.nvls import nvls_supported
    if not nvls_supported(0):
        pytest.skip("no NVLink multicast on this machine")
    rep = run_fanout("tiny-llama", "nvls", [dict(tp=1)], dict(tp=1), ["cuda:0"], ["cuda:0", "cuda:1"])
    assert rep[0]["mc_groups"] == 1 and rep[0]["mc_items"] > 0


def test_nvls_fanout_tp2_trainer_multicasts_from_both_ranks():
    """TP2 trainer into two TP1 replicas by multicast: the layer norms both TP ranks hold go to
    both replicas from the same rank (replica-consistent assignment), so each rank writes the
    same entries to both replicas and joins the multicast group."""
    _need(4)
    from tests.e2e_harness import run_fanout
    from weightbridge_b200.parallel.nvls import nvls_supported
    if not nvls_supported(0):
        pytest.skip("no NVLink multicast on this machine")
    rep = run_fanout("tiny-llama", "nvls", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1),
                     ["cuda:0", "cuda:1"], ["cuda:2", "cuda:3"])
    assert all(r["mc_groups"] == 1 and r["mc_items"] > 0 for r in rep.values()), rep


def test_data_parallel_trainer_serves_the_worker_on_its_gpu():
    """Two identical trainer ranks (DP 2) on GPUs 0 and 1, a TP1 worker beside each: every entry
    reaches a worker from the rank on its own GPU (an HBM copy), none over NVLink."""
    _need(2)
    from tests.e2e_harness import run_fanout
    rep = run_fanout("tiny-llama", "gpu_direct", [dict(tp=1), dict(tp=1)], dict(tp=1), ["cuda:0", "cuda:1"],
                     ["cuda:0", "cuda:1"])
    assert rep[0]["targets"] == [2] and rep[1]["targets"] == [3], rep
