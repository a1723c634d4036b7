"""The control-plane latency tool runs and reports every field."""
from weightbridge_b200.control.latency import measure


def test_latency_tool_direct_arm():
    r = measure("direct", syncs=24)
    assert r["payload_bytes"] > 0
    assert all(r[k] is not None and r[k] > 0 for k in ("send_ms", "wait_ready_ms", "copy_ms", "request_update_ms"))


def test_latency_tool_pull_direction():
    """Pulling, the worker runs the copy and the sender waits for no ready key."""
    r = measure("direct", syncs=24, direction="pull")
    assert r["direction"] == "pull" and r["payload_bytes"] > 0
    assert r["send_ms"] > 0 and r["request_update_ms"] > 0 and r["wait_ready_ms"] == 0
