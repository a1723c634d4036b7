"""Planner + C++ CPU executor: direct (address to address) and wire (pack / unpack) paths."""
import numpy as np
import pytest
import torch

from weightbridge_b200 import WeightData
from weightbridge_b200.core.binding import bind
from weightbridge_b200.core.plan import (ITEM_DTYPE, lower_ops, phys_binding, plan_pair, wire_binding,
                                         plan_digest)
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.ops.executor import cpu_execute, cpu_piece_amax
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout

ABS = lambda _alloc: 0   # alloc -1: offsets are absolute addresses


def _u8(t):
    return t.view(torch.uint8) if t.dtype in (torch.float8_e4m3fn,) else t


def make_senders(layouts, dtype):
    out = []
    for lay in layouts:
        params = lay.allocate(dtype=dtype)
        meta, views = lay.to_wb(params)
        out.append((params, meta, phys_binding(bind(meta, views))))
    return out


def make_receiver(lay, dtype):
    params = lay.allocate(dtype=dtype)
    meta, views = lay.to_wb(params)
    return params, meta, phys_binding(bind(meta, views))


CASES = [
    ("tiny-llama", [dict(tp=2, tp_rank=i) for i in range(2)], [dict(tp=1)], torch.float32),
    ("tiny-llama", [dict(pp=2, pp_rank=i) for i in range(2)], [dict(tp=4, tp_rank=i) for i in range(4)], torch.bfloat16),
    ("tiny-qwen2", [dict(tp=2, tp_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i) for i in range(2)], torch.bfloat16),
    ("tiny-qwen3-moe", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i) for i in range(2)], torch.bfloat16),
    ("tiny-mixtral", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=1)], torch.bfloat16),
]


@pytest.mark.parametrize("model,meg,sgl,dtype", CASES)
@pytest.mark.parametrize("item_bytes", [1 << 19, 4096])
def test_direct_plan_cpu_executor(model, meg, sgl, dtype, item_bytes):
    arch = get_arch(model)
    senders = make_senders([MegatronLayout(arch, **m) for m in meg], dtype)
    for s in sgl:
        lay = SGLangLayout(arch, **s)
        params, meta, rphys = make_receiver(lay, dtype)
        for _p, _m, sphys in senders:
            ops = plan_pair(sphys, rphys)
            tables = lower_ops(ops, ABS, ABS, item_bytes=item_bytes)
            assert tables.items.dtype == ITEM_DTYPE
            if item_bytes == 4096:
                assert all(int(r) * int(b) <= 4096 or int(r) == 1 for r, b in zip(tables.items["rows"], tables.items["row_bytes"]))
            cpu_execute(tables)
        expected = lay.allocate(dtype=dtype, fill=True)
        for n in params:
            assert torch.equal(params[n], expected[n]), n


def test_wire_path_roundtrip():
    """sender -> packed wire (overlap order) -> receiver, as the gloo path does."""
    arch = get_arch("tiny-llama")
    senders = make_senders([MegatronLayout(arch, tp=2, tp_rank=i) for i in range(2)], torch.float32)
    lay = SGLangLayout(arch, tp=1)
    params, rmeta, rphys = make_receiver(lay, torch.float32)
    for _p, smeta, sphys in senders:
        ov = WeightData.compute_overlap(smeta, rmeta)
        wire = torch.empty(ov.total_nbytes(), dtype=torch.uint8)
        wb = wire_binding(ov, base=wire.data_ptr())
        cpu_execute(lower_ops(plan_pair(sphys, wb, overlap_meta=ov), ABS, ABS))
        cpu_execute(lower_ops(plan_pair(wb, rphys), ABS, ABS))
        # the wire buffer equals the reference-compatible host packer's output
        ref = WeightData.pack_for(smeta, {k: v for k, v in zip(*_views_of(smeta, _p))}, ov)
        assert torch.equal(ref, wire)
    expected = lay.allocate(dtype=torch.float32, fill=True)
    for n in params:
        assert torch.equal(params[n], expected[n]), n


def _views_of(meta, params):
    lay = MegatronLayout(get_arch("tiny-llama"), tp=2, tp_rank=0)
    names = []
    views = []
    # rebuild the views from params (same layout object semantics)
    for r in range(2):
        lay = MegatronLayout(get_arch("tiny-llama"), tp=2, tp_rank=r)
        m, v = lay.to_wb(params)
        if m == meta:
            return list(v.keys()), list(v.values())
    raise AssertionError("no matching layout")


def test_cast_fp32_to_bf16():
    arch = get_arch("tiny-llama")
    senders = make_senders([MegatronLayout(arch, tp=2, tp_rank=i) for i in range(2)], torch.float32)
    lay = SGLangLayout(arch, tp=2, tp_rank=1)
    params, _m, rphys = make_receiver(lay, torch.bfloat16)
    for _p, _sm, sphys in senders:
        ops = plan_pair(sphys, rphys)
        assert {o.kind for o in ops} == {"cast"}
        cpu_execute(lower_ops(ops, ABS, ABS))
    expected = {k: v.to(torch.bfloat16) for k, v in lay.allocate(dtype=torch.float32, fill=True).items()}
    for n in params:
        assert torch.equal(params[n], expected[n]), n


def test_fp8_quant_plan_cpu():
    arch = get_arch("tiny-qwen3-moe")
    senders = make_senders([MegatronLayout(arch, ep=2, ep_rank=i) for i in range(2)], torch.bfloat16)
    for r in range(2):
        lay = SGLangLayout(arch, tp=2, tp_rank=r, moe_ep=2, quant="fp8_experts")
        params, _m, rphys = make_receiver(lay, torch.bfloat16)
        kinds = set()
        for _p, _sm, sphys in senders:
            ops = plan_pair(sphys, rphys)
            kinds |= {o.kind for o in ops}
            t = lower_ops(ops, ABS, ABS)
            cpu_execute(t)
        assert "quant" in kinds
        expected = lay.allocate(dtype=torch.bfloat16, fill=True)
        for n in params:
            assert torch.equal(_u8(params[n]), _u8(expected[n])), n


def test_plan_digest_is_deterministic():
    arch = get_arch("tiny-llama")
    (_, _, s0), = make_senders([MegatronLayout(arch, tp=1)], torch.float32)
    _, rmeta, rphys = make_receiver(SGLangLayout(arch, tp=2, tp_rank=0), torch.float32)
    assert plan_digest(plan_pair(s0, rphys)) == plan_digest(plan_pair(s0, rphys))
    ov = WeightData.compute_overlap(s0.meta, rmeta)
    assert plan_digest(ov) == plan_digest(WeightData(bytes(ov)))


def test_validate_tables_catches_out_of_bounds_rows():
    from weightbridge_b200.core.plan import Op, PlanBoundsError, storage_ranges, validate_tables
    a = torch.arange(64, dtype=torch.float32)
    b = torch.zeros(32, dtype=torch.float32)
    good = Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [32], [1], [1], a.dtype, a.dtype)
    t = lower_ops([good], ABS, ABS)
    validate_tables(t, storage_ranges([a]), storage_ranges([b]))
    over = Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr() + 4), [32], [1], [1], a.dtype, a.dtype)
    with pytest.raises(PlanBoundsError, match="write"):
        validate_tables(lower_ops([over], ABS, ABS), storage_ranges([a]), storage_ranges([b]))
    rd = Op("copy", "x", (-1, a.data_ptr() + 40 * 4), (-1, b.data_ptr()), [32], [1], [1], a.dtype, a.dtype)
    with pytest.raises(PlanBoundsError, match="read"):
        validate_tables(lower_ops([rd], ABS, ABS), storage_ranges([a]), storage_ranges([b]))
    # 2-D rows: the last row's end is what matters
    m = torch.zeros(8, 16)
    o2 = Op("copy", "x", (-1, a.data_ptr()), (-1, m.data_ptr() + 4), [8, 8], [8, 1], [16, 1], a.dtype, a.dtype)
    validate_tables(lower_ops([o2], ABS, ABS), storage_ranges([a]), storage_ranges([m]))
    o3 = Op("copy", "x", (-1, a.data_ptr()), (-1, m.data_ptr() + 36 * 4), [8, 8], [8, 1], [16, 1], a.dtype, a.dtype)
    with pytest.raises(PlanBoundsError):
        validate_tables(lower_ops([o3], ABS, ABS), storage_ranges([a]), storage_ranges([m]))


@pytest.mark.parametrize("model,meg,sgl", [c[:3] for c in CASES])
def test_real_plans_validate(model, meg, sgl):
    from weightbridge_b200.core.plan import storage_ranges, validate_tables
    arch = get_arch(model)
    dtype = torch.bfloat16
    for m in meg:
        lay = MegatronLayout(arch, **m)
        params = lay.allocate(dtype=dtype)
        smeta, sviews = lay.to_wb(params)
        sphys = phys_binding(bind(smeta, sviews))
        for s in sgl:
            rl = SGLangLayout(arch, **s)
            rparams = rl.allocate(dtype=dtype, pool=True)
            rmeta, rviews = rl.to_wb(rparams)
            t = lower_ops(plan_pair(sphys, phys_binding(bind(rmeta, rviews))), ABS, ABS)
            validate_tables(t, storage_ranges(params.values()), storage_ranges(rparams.values()))


def test_multicast_lowering_rules():
    from weightbridge_b200.core.plan import OP_COPY_MC, Op, multicast_ok
    a = torch.zeros(64, dtype=torch.bfloat16)
    ok = Op("copy", "x", (-1, 0), (0, 256), [64], [1], [1], torch.bfloat16, torch.bfloat16)
    assert multicast_ok(ok, lambda x: a.data_ptr() // 16 * 16, lambda x: 1 << 20)
    t = lower_ops([ok], lambda x: 4096, lambda x: 1 << 20, multicast=True)
    assert ((t.items["op"] & 0xFF) == OP_COPY_MC).all()
    odd = Op("copy", "x", (-1, 2), (0, 256), [64], [1], [1], torch.bfloat16, torch.bfloat16)
    assert not multicast_ok(odd, lambda x: 4096, lambda x: 1 << 20)
    cast = Op("cast", "x", (-1, 0), (0, 0), [64], [1], [1], torch.float32, torch.bfloat16)
    assert not multicast_ok(cast, lambda x: 4096, lambda x: 1 << 20)
    with pytest.raises(ValueError):
        lower_ops([cast], lambda x: 0, lambda x: 0, multicast=True)
    q = Op("quant", "x", (-1, 0), (0, 0), [128, 128], [128, 1], [128, 1], torch.bfloat16, torch.float8_e4m3fn,
           (0, 0), [1, 1], (128, 128))
    with pytest.raises(ValueError):
        lower_ops([q], lambda x: 0, lambda x: 0, multicast=True)


def test_data_ptrs_key_detects_rebinding():
    """The sender's binding key: equal for the same tensors, different when a tensor (or a
    view inside a multi-shard list) is replaced."""
    from weightbridge_b200.ops._ext import ext
    a, b, c = torch.zeros(4), torch.zeros(4), torch.zeros(4)
    k1 = ext().data_ptrs([a, [a, b]])
    assert k1 == ext().data_ptrs([a, [a, b]])
    assert k1 != ext().data_ptrs([a, [a, c]])
    assert k1 != ext().data_ptrs([a, [a], b])
    assert len(ext().data_ptrs([None, a[1:]])) == 16


def test_mixtral_fp8_experts_plan_cpu():
    """Mixtral names (block_sparse_moe, w1/w3/w2) through the fp8 expert path."""
    arch = get_arch("tiny-mixtral")
    senders = make_senders([MegatronLayout(arch, ep=2, ep_rank=i) for i in range(2)], torch.bfloat16)
    lay = SGLangLayout(arch, tp=1, quant="fp8_experts")
    params, meta, rphys = make_receiver(lay, torch.bfloat16)
    assert any(".block_sparse_moe.experts.3.w2.weight" in n for n in meta.names())
    for _p, _sm, sphys in senders:
        cpu_execute(lower_ops(plan_pair(sphys, rphys), ABS, ABS))
    expected = lay.allocate(dtype=torch.bfloat16, fill=True)
    for n in params:
        assert torch.equal(_u8(params[n]), _u8(expected[n])), n


def test_mixtral_from_hf_config():
    from weightbridge_b200.models.arch import ModelArch
    a = ModelArch.from_hf_config({"model_type": "mixtral", "hidden_size": 4096, "num_attention_heads": 32,
                                  "num_key_value_heads": 8, "num_hidden_layers": 32, "intermediate_size": 14336,
                                  "vocab_size": 32000, "num_local_experts": 8, "num_experts_per_tok": 2})
    assert a == get_arch("mixtral-8x7b").with_(name="mixtral")


@pytest.mark.parametrize("quant", ["fp8_experts", "fp8_linear"])
def test_qwen2_moe_shared_expert_fp8_plan_cpu(quant):
    """Qwen2-MoE: routed experts, the gated shared expert (a TP-split dense MLP) and q/k/v
    bias; fp8 on the experts only or on every linear layer."""
    arch = get_arch("tiny-qwen2-moe")
    senders = make_senders([MegatronLayout(arch, tp=2, tp_rank=i) for i in range(2)], torch.bfloat16)
    lay = SGLangLayout(arch, tp=1, quant=quant)
    params, meta, rphys = make_receiver(lay, torch.bfloat16)
    assert "model.layers.1.mlp.shared_expert.gate_up_proj.weight" in params
    # fp8_linear: k/v of one 64-row KV group are half a block, so blocks span the two TP ranks
    tables = [lower_ops(plan_pair(sphys, rphys), ABS, ABS, receiver=0) for _p, _sm, sphys in senders]
    assert (quant == "fp8_linear") == any(len(t.pieces) for t in tables)
    block = {}
    for t in tables:
        for k, a in zip(t.piece_keys, cpu_piece_amax(t)):
            block[k] = max(block.get(k, 0.0), float(a))
    for t in tables:
        cpu_execute(t, np.array([block[k] for k in t.piece_keys], dtype=np.float32))
    expected = lay.allocate(dtype=torch.bfloat16, fill=True)
    for n in params:
        assert torch.equal(_u8(params[n]), _u8(expected[n])), n


def test_qwen2_moe_from_hf_config():
    from weightbridge_b200.models.arch import ModelArch
    a = ModelArch.from_hf_config({"model_type": "qwen2_moe", "hidden_size": 2048, "num_attention_heads": 16,
                                  "num_key_value_heads": 16, "num_hidden_layers": 24, "intermediate_size": 5632,
                                  "moe_intermediate_size": 1408, "shared_expert_intermediate_size": 5632,
                                  "vocab_size": 151936, "num_experts": 60, "num_experts_per_tok": 4})
    assert a.family == "qwen2_moe" and a.ffn == 0 and a.shared_ffn == 5632 and a.qkv_bias and a.is_moe


def test_pack_for_fp8_linear_from_grouped_qkv():
    """The host pack path (WeightData.pack_for) on refined-row regions whose groups hold whole
    blocks (128-row KV heads): the same bytes as quantising the whole tensors."""
    from weightbridge_b200.core.binding import unpack_from
    arch = get_arch("tiny-llama-fp8")
    r = SGLangLayout(arch, tp=1, quant="fp8_linear")
    rp = r.allocate(dtype=torch.bfloat16)
    rm, rv = r.to_wb(rp)
    for i in range(2):
        s = MegatronLayout(arch, tp=2, tp_rank=i)
        sp = s.allocate(dtype=torch.bfloat16)
        sm, sv = s.to_wb(sp)
        ov = WeightData.compute_overlap(sm, rm)
        unpack_from(bind(rm, rv), ov, WeightData.pack_for(sm, sv, ov))
    exp = r.allocate(dtype=torch.bfloat16, fill=True)
    assert all(torch.equal(_u8(rp[n]), _u8(exp[n])) for n in exp)


@pytest.mark.parametrize("quant", [None, "fp8_experts"])
def test_redundant_expert_slots(quant):
    """SGLang EPLB-style placement: physical slots naming logical experts, one of them twice
    (and a per-layer map): every slot receives its expert, the duplicate included, with its
    own block scales under fp8."""
    arch = get_arch("tiny-qwen3-moe")
    senders = make_senders([MegatronLayout(arch, ep=2, ep_rank=i) for i in range(2)], torch.bfloat16)
    slots = [[0, 5, 2, 5, 7], [1, 1, 3, 6, 4]]          # layer 0, layer 1
    lay = SGLangLayout(arch, tp=1, quant=quant, expert_slots=slots)
    params, meta, rphys = make_receiver(lay, torch.bfloat16)
    assert params["model.layers.0.mlp.experts.w13_weight"].shape[0] == 5
    assert len(meta.shards("model.layers.0.mlp.experts.5.gate_proj.weight")) == 2
    for _p, _sm, sphys in senders:
        cpu_execute(lower_ops(plan_pair(sphys, rphys), ABS, ABS))
    expected = lay.allocate(dtype=torch.bfloat16, fill=True)
    for n in params:
        assert torch.equal(_u8(params[n]), _u8(expected[n])), n
    w = params["model.layers.0.mlp.experts.w13_weight"]
    assert torch.equal(_u8(w[1]), _u8(w[3]))                # both slots of expert 5
    if quant:
        sc = params["model.layers.0.mlp.experts.w13_weight_scale_inv"]
        assert torch.equal(sc[1], sc[3]) and not torch.equal(sc[0], sc[1])


def _transpose_case(dtype, lead, R, C, src_off=0, dst_off=0, device="cpu"):
    """A copy of ``[lead, R, C]`` (rows contiguous) into a destination that stores each
    ``[R, C]`` matrix column-major (MLA's w_kc against kv_b_proj); offsets misalign rows."""
    from weightbridge_b200.core.plan import Op
    base = torch.arange(lead * R * C + src_off, dtype=torch.float64, device=device).to(dtype) \
        if dtype.is_floating_point else torch.randint(0, 100, (lead * R * C + src_off,), device=device).to(dtype)
    src = base[src_off:].view(lead, R, C)
    dst_store = torch.zeros(lead * C * R + dst_off, dtype=dtype, device=device)
    dst = dst_store[dst_off:].view(lead, C, R).transpose(1, 2)       # logical [lead, R, C]
    es = src.element_size()
    op = Op("copy", "w", (-1, src.data_ptr()), (-1, dst.data_ptr()), [lead, R, C], list(src.stride()),
            list(dst.stride()), dtype, dtype)
    return op, src, dst, dst_store, es


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.uint8])
def test_transposed_destination_lowers_to_tiled_transposes(dtype):
    """A destination contiguous along the source's rows lowers to OP_TRANSPOSE work rows (one
    per matrix and column chunk), which the C++ executor writes exactly; the bounds check
    covers the destination rows a transpose writes."""
    from weightbridge_b200.core.plan import OP_TRANSPOSE, PlanBoundsError, validate_tables
    op, src, dst, store, es = _transpose_case(dtype, 3, 70, 130, src_off=1, dst_off=3)
    t = lower_ops([op], ABS, ABS, item_bytes=64 * 70 * es)
    assert len(t.items) == 3 * 3 and ((t.items["op"] & 0xFF) == OP_TRANSPOSE).all()
    srange = [(src.data_ptr(), src.data_ptr() + src.numel() * es)]
    drange = [(store.data_ptr(), store.data_ptr() + store.numel() * es)]
    validate_tables(t, srange, drange)
    with pytest.raises(PlanBoundsError):
        validate_tables(t, srange, [(drange[0][0], drange[0][1] - es)])
    cpu_execute(t)
    assert torch.equal(dst, src)
    assert not store[:3].to(torch.float32).any()


def test_interleave_deals_items_and_blocks_round_robin():
    """Per-peer tables are merged so that consecutive copy items and consecutive quantised
    blocks go to different peers (no peer's work all comes first), every row kept once."""
    import numpy as np
    from weightbridge_b200.control.sender import _interleave
    from weightbridge_b200.core.plan import ITEM_DTYPE, QDESC_DTYPE, QWORK_DTYPE, Tables
    parts = []
    for p, (ni, nq) in enumerate([(5, 4), (2, 6), (3, 0)]):
        it = np.zeros(ni, ITEM_DTYPE)
        it["dst"] = 1000 * p + np.arange(ni)
        qd = np.zeros(1 if nq else 0, QDESC_DTYPE)
        qw = np.zeros(nq, QWORK_DTYPE)
        qw["block"] = 1000 * p + np.arange(nq)
        parts.append(Tables(it, qd, qw))
    t = _interleave(parts)
    assert list(t.items["dst"] // 1000)[:6] == [0, 1, 2, 0, 1, 2]
    assert sorted(t.items["dst"].tolist()) == sorted(np.concatenate([p.items["dst"] for p in parts]).tolist())
    peers = (t.qwork["block"] // 1000).tolist()
    assert peers[:4] == [0, 1, 0, 1] and sorted(t.qwork["block"].tolist()) == [0, 1, 2, 3] + [1000 + i for i in range(6)]
    # each block still points at its own peer's descriptor
    assert all(int(d) == (0 if b < 1000 else 1) for d, b in zip(t.qwork["desc"], t.qwork["block"]))
