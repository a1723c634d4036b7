"""Chunked wires of the wire modes: the cut (core/wire.py) and the double-buffered transfer
(control/wires.py) over gloo with many chunks per peer."""
import torch

from weightbridge_b200.core.shard import WeightData
from weightbridge_b200.core.wire import wire_chunks
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout


def _overlap(quant=None):
    a = get_arch("tiny-qwen3-moe")
    s = MegatronLayout(a, ep=2, ep_rank=0)
    r = SGLangLayout(a, tp=1, quant=quant)
    sm, _ = s.to_wb(s.allocate(fill=False))
    rm, _ = r.to_wb(r.allocate(fill=False))
    return WeightData.compute_overlap(sm, rm)


def test_chunks_keep_order_sizes_and_scale_pairs():
    ov = _overlap("fp8_experts")
    limit = 150_000
    chunks = wire_chunks(ov, limit)
    assert len(chunks) > 5
    assert [n for c in chunks for n in c.names()] == ov.names()
    assert sum(c.total_nbytes() for c in chunks) == ov.total_nbytes()
    for c in chunks:
        names = c.names()
        for n in names:
            q = c.quant(n)
            if q and q.get("role") != "scale":
                assert q["scale"] in names          # the pack writes weight and scale together
        if len(names) > 2:
            assert c.total_nbytes() <= limit
    assert len(wire_chunks(ov, 0)) == 1
    assert len(wire_chunks(ov, 1)) == len([n for n in ov.names() if not n.endswith("_scale_inv")])


def test_chunked_gloo_sync_tp2_to_tp1():
    """48 KiB chunks: every pair moves many messages through two buffers."""
    from tests.e2e_harness import run
    run("tiny-llama", "cpu_direct", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], dict(tp=1), n_syncs=2,
        cfg_extra={"wire_chunk_bytes": 48 << 10})


def test_chunked_gloo_sync_split_fp8_blocks():
    """Chunks and split fp8 blocks together: the amax pass covers the pieces of every chunk."""
    from tests.e2e_harness import run
    run("tiny-qwen3-moe", "cpu_direct", [dict(etp=4, etp_rank=i) for i in range(4)],
        dict(tp=1, quant="fp8_experts"), dtype=torch.bfloat16, n_syncs=2, cfg_extra={"wire_chunk_bytes": 64 << 10})


from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=200, deadline=None)
@given(sizes=st.lists(st.integers(1, 5000), min_size=1, max_size=12), chunk=st.integers(0, 8000),
       pick=st.lists(st.booleans(), min_size=12, max_size=12))
def test_buffer_size_holds_every_chunk_of_every_subset(sizes, chunk, pick):
    """The wire sets of partial syncs reuse the full sync's buffers: a buffer of
    buffer_bytes(full overlap) holds every chunk of any subset of its entries."""
    import torch
    from weightbridge_b200 import WeightData
    from weightbridge_b200.core.wire import buffer_bytes, restrict_overlap, wire_chunks
    ov = WeightData({f"e{i}": {"shard": [(0, n, n)], "dtype": torch.uint8} for i, n in enumerate(sizes)})
    cap = buffer_bytes(ov, chunk)
    names = [f"e{i}" for i in range(len(sizes)) if pick[i]] or ["e0"]
    for sub in (ov, restrict_overlap(ov, names)):
        assert all(c.total_nbytes() <= cap for c in wire_chunks(sub, chunk))
