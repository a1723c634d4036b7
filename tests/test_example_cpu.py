"""The examples run end to end on CPU (gloo path)."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_single_node_example_cpu():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "examples", "single_node.py"), "--device", "cpu",
                          "--steps", "2", "--workers", "2"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "all syncs verified" in out.stdout


def test_single_node_example_fsdp_trainer_cpu():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "examples", "single_node.py"), "--device", "cpu",
                          "--steps", "2", "--workers", "2", "--trainers", "3", "--trainer", "fsdp"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "all syncs verified" in out.stdout


def test_raw_shards_example_cpu():
    """The reference example's scenario: uneven row split, column split and a duplicated
    tensor on two trainer ranks, two rollout workers holding row halves in flat buffers."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "examples", "raw_shards.py"), "--device", "cpu",
                          "--steps", "2"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert out.stdout.strip().splitlines()[-1].startswith("OK")


def test_single_node_example_fsdp_trainer_into_mla_workers_cpu():
    """Three FSDP ranks (row ranges that end inside attention heads) into two SGLang workers of
    a DeepSeek-style model: kv_b_proj with its derived w_kc / w_vc."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "examples", "single_node.py"), "--device", "cpu",
                          "--steps", "1", "--workers", "2", "--trainers", "3", "--trainer", "fsdp",
                          "--model", "tiny-deepseek-v3"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "all syncs verified" in out.stdout
