"""Public API on one GPU: trainer and rollout in separate processes, colocated on cuda:0,
receiver memory mapped into the senders with CUDA IPC, the sm_100a kernel moving the data.
No kernel waits on another process's kernel (completion goes through the session store)."""
import pytest
import torch

from tests.e2e_harness import run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("direction", ["pull", "push"])
def test_colocated_ipc_tiny_llama_tp2_to_tp1(direction):
    run("tiny-llama", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1),
        device="cuda:0", dtype=torch.bfloat16, direction=direction)


@pytest.mark.parametrize("direction", ["pull", "push"])
def test_colocated_ipc_qwen3_moe_fp8_experts(direction):
    """pull: the receiver loads the bf16 copies while the senders quantise and push the fp8
    expert blocks; push: the senders store everything."""
    run("tiny-qwen3-moe", "gpu_direct", [dict(ep=2, ep_rank=0), dict(ep=2, ep_rank=1)],
        dict(tp=1, quant="fp8_experts"), device="cuda:0", dtype=torch.bfloat16, n_syncs=2, direction=direction)


def test_colocated_ipc_reference_style_late_binding():
    """Receiver created with metadata only; tensors handed over at request_update."""
    run("tiny-qwen3", "gpu_direct", [dict(tp=1)], dict(tp=2, tp_rank=1), device="cuda:0",
        dtype=torch.bfloat16, late=True)


def test_colocated_ipc_split_fp8_blocks():
    """Expert TP 4 (64-row slices): every expert block is split over two senders, which
    exchange the block amax through the session before their kernels store into the
    receiver's fp8 weights over CUDA IPC."""
    run("tiny-qwen3-moe", "gpu_direct", [dict(etp=4, etp_rank=i) for i in range(4)],
        dict(tp=1, quant="fp8_experts"), device="cuda:0", dtype=torch.bfloat16, n_syncs=2)


def test_colocated_ipc_fp8_linear_from_grouped_qkv():
    """fp8 on every linear layer from Megatron TP 2: grouped-QKV overlaps cut per KV group,
    K/V blocks split between the two ranks (amax exchanged), stores over CUDA IPC."""
    run("tiny-qwen2-moe", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)],
        dict(tp=1, quant="fp8_linear"), device="cuda:0", dtype=torch.bfloat16, n_syncs=2)


def test_colocated_ipc_pull_direction():
    """The receiver maps the senders' memory (CUDA IPC) and runs the pull kernel itself."""
    run("tiny-llama", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1),
        device="cuda:0", dtype=torch.bfloat16, direction="pull")


def test_raw_shards_example_on_one_gpu():
    """Hand-built metadata (uneven rows, column split, duplicated tensor), flat receiver
    buffers bound at request_update, two trainer and two worker processes on cuda:0."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "examples", "raw_shards.py"), "--device", "cuda",
                          "--steps", "2"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert out.stdout.strip().splitlines()[-1].startswith("OK")


def test_inprocess_send_async_on_gpu():
    """Sender, controller and receiver in one process on cuda:0 (the sender uses the
    receiver's addresses directly); send_async overlaps with the caller and tags the weights."""
    import threading
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout
    torch.cuda.set_device(0)
    arch = get_arch("tiny-llama")
    cfg = TransferConfig(mode="gpu_direct", connect_timeout_s=60, sync_timeout_s=60)
    with WeightReceiverController(worker_num=1, timeout_s=30) as ctl:
        url = ctl.serve()
        rl = SGLangLayout(arch, tp=1)
        rp = rl.allocate(device="cuda:0", dtype=torch.bfloat16)
        rm, rv = rl.to_wb(rp)
        with WeightReceiver(ctl.ipc_name, 0, rm, state_dict=rv, config=cfg) as recv:
            sl = MegatronLayout(arch, tp=1)
            sp = sl.allocate(device="cuda:0", dtype=torch.bfloat16, seed=3)
            sm, sv = sl.to_wb(sp)
            with WeightSender("gpu_direct", [url], config=cfg) as s:
                s.connect(sm)
                th = threading.Thread(target=lambda: recv.request_update(timeout=30))
                th.start()
                st = s.send_async(sv, version=3).result(timeout=60)
                th.join(30)
                assert st.status == 0 and recv.weights_version == 3
    exp = rl.allocate(device="cuda:0", dtype=torch.bfloat16, fill=True, seed=3)
    assert all(torch.equal(rp[n], exp[n]) for n in exp)


def test_inprocess_send_async_snapshot_on_gpu():
    """send_async(snapshot=True) on cuda:0: the copy is enqueued on the caller's stream, the
    caller overwrites its parameters right away (the next optimizer step) and the worker
    still receives the values of the call."""
    import threading
    from weightbridge_b200 import TransferConfig, WeightReceiver, WeightReceiverController, WeightSender
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout
    torch.cuda.set_device(0)
    arch = get_arch("tiny-llama")
    cfg = TransferConfig(mode="gpu_direct", connect_timeout_s=60, sync_timeout_s=60)
    with WeightReceiverController(worker_num=1, timeout_s=30) as ctl:
        url = ctl.serve()
        rl = SGLangLayout(arch, tp=1)
        rp = rl.allocate(device="cuda:0", dtype=torch.bfloat16)
        rm, rv = rl.to_wb(rp)
        with WeightReceiver(ctl.ipc_name, 0, rm, state_dict=rv, config=cfg) as recv:
            sl = MegatronLayout(arch, tp=1)
            sp = sl.allocate(device="cuda:0", dtype=torch.bfloat16, seed=3)
            sm, sv = sl.to_wb(sp)
            with WeightSender("gpu_direct", [url], config=cfg) as s:
                s.connect(sm)
                th = threading.Thread(target=lambda: recv.request_update(timeout=30))
                th.start()
                fut = s.send_async(sv, version=4, snapshot=True)
                torch._foreach_add_(list(sp.values()), 1.0)
                st = fut.result(timeout=60)
                th.join(30)
                assert st.status == 0 and recv.weights_version == 4
    exp = rl.allocate(device="cuda:0", dtype=torch.bfloat16, fill=True, seed=3)
    assert all(torch.equal(rp[n], exp[n]) for n in exp)


def test_colocated_ipc_deepseek_mla_fp8_experts():
    """DeepSeek-style model from Megatron TP 2 over CUDA IPC: MLA with the worker's derived
    w_kc / w_vc (transposed strided destinations), dense first layer, shared experts, router
    bias, fp8 routed experts."""
    run("tiny-deepseek-v3", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)],
        dict(tp=1, quant="fp8_experts"), device="cuda:0", dtype=torch.bfloat16, n_syncs=2)


def test_colocated_ipc_partial_syncs_with_split_fp8_blocks():
    """Odd syncs send layer 1 only (names=): the split K/V fp8 blocks of that layer are
    quantised with the exchanged amax, the other layers keep the previous weights."""
    run("tiny-qwen2-moe", "gpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)],
        dict(tp=1, quant="fp8_linear"), device="cuda:0", dtype=torch.bfloat16, n_syncs=3,
        subset_prefix="model.layers.1.")
