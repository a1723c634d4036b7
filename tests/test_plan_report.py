"""The dry-run planner report (meta tensors only)."""
import json
import subprocess
import sys

from weightbridge_b200.plan_report import report


def test_report_tiny_llama_tp2_to_two_replicas():
    rep = report("tiny-llama", {"tp": 2}, {"tp": 1}, replicas=2)
    assert len(rep["senders"]) == 2 and len(rep["receivers"]) == 2
    # every replica receives the whole model once
    per_replica = {r["receiver"]: r["ingress_bytes"] for r in rep["receivers"]}
    assert per_replica[0] == per_replica[1] == rep["total_written_bytes"] // 2
    assert rep["link_bound_ms"] > 0


def test_report_counts_split_pieces_for_expert_tp4_fp8():
    rep = report("tiny-qwen3-moe", {"etp": 4}, {"tp": 1, "quant": "fp8_experts"})
    assert all(s["split_pieces"] > 0 for s in rep["senders"])
    rep2 = report("tiny-qwen3-moe", {"ep": 2}, {"tp": 1, "quant": "fp8_experts"})
    assert all(s["split_pieces"] == 0 and s["quant_blocks"] > 0 for s in rep2["senders"])


def test_report_cli_json():
    out = subprocess.run([sys.executable, "-m", "weightbridge_b200.plan_report", "--model", "tiny-qwen3",
                          "--trainer", "tp=2", "--rollout", "tp=2", "--json"],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    rep = json.loads(out.stdout)
    assert rep["model"] == "tiny-qwen3" and len(rep["senders"]) == 2


def test_report_fsdp_trainer_counts_split_pieces():
    rep = report("tiny-llama-fp8", {"world": 3}, {"tp": 1, "quant": "fp8_linear"}, trainer_kind="fsdp")
    assert len(rep["senders"]) == 3 and sum(s["split_pieces"] for s in rep["senders"]) > 0
