"""Coverage checks: receivers are poisoned (NaN) before a sync; afterwards no bound element
may still hold the poison, and padding outside the bound entries must still hold it (nothing
writes where it should not).  Random layout pairs come from Hypothesis."""
import torch
from hypothesis import given, settings, strategies as st

from weightbridge_b200.core.binding import bind
from weightbridge_b200.core.plan import lower_ops, phys_binding, plan_pair
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.ops.executor import cpu_execute
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout

ABS = lambda _a: 0


def _sync(arch, megs, sgl, dtype=torch.float32):
    senders, keep = [], []          # keep: physical bindings hold addresses, not references
    for m in megs:
        lay = MegatronLayout(arch, **m)
        p = lay.allocate(dtype=dtype)
        meta, views = lay.to_wb(p)
        keep.append(p)
        senders.append(phys_binding(bind(meta, views)))
    rl = SGLangLayout(arch, **sgl)
    rp = rl.allocate(dtype=dtype, pool=True)
    for t in rp.values():           # poison every parameter, padding included (0xFF.. is a NaN)
        t.view(torch.uint8).fill_(0xFF)
    rmeta, rviews = rl.to_wb(rp)
    rphys = phys_binding(bind(rmeta, rviews))
    for sp in senders:
        cpu_execute(lower_ops(plan_pair(sp, rphys), ABS, ABS, item_bytes=4096))
    return rl, rp, rmeta, rviews


def _all_ranks(cfg, key_rank, n):
    return [dict(cfg, **{key_rank: i}) for i in range(n)]


@settings(max_examples=25, deadline=None)
@given(model=st.sampled_from(["tiny-llama", "tiny-qwen2", "tiny-qwen3"]),
       mtp=st.sampled_from([1, 2]), mpp=st.sampled_from([1, 2]),
       rtp=st.sampled_from([1, 2, 4]), attn_dp=st.booleans(), rrank=st.integers(0, 3))
def test_random_dense_layouts_cover_exactly(model, mtp, mpp, rtp, attn_dp, rrank):
    arch = get_arch(model)
    if arch.num_kv_heads % mtp or (arch.num_kv_heads < rtp and rtp % arch.num_kv_heads):
        return
    megs = [dict(tp=mtp, pp=mpp, tp_rank=t, pp_rank=p) for t in range(mtp) for p in range(mpp)]
    sgl = dict(tp=rtp, tp_rank=rrank % rtp)
    if attn_dp:
        sgl.update(attn_tp=1, attn_tp_rank=0)
    rl, rp, rmeta, rviews = _sync(arch, megs, sgl)
    exp = rl.allocate(dtype=torch.float32, fill=True)
    for name, v in rviews.items():
        assert not torch.isnan(v).any(), f"{name} not fully written"
    for n in rp:
        # padding rows (vocab padding) keep the poison; everything bound matches the oracle
        if "embed_tokens" in n or "lm_head" in n:
            V = arch.vocab
            rows = rl.padded_vocab // rl.tp
            l = rl.tp_rank * rows
            valid = max(0, min(rows, V - l))
            assert torch.equal(rp[n][:valid], exp[n][:valid])
            assert torch.isnan(rp[n][valid:]).all()
        else:
            assert torch.equal(rp[n], exp[n]), n


@settings(max_examples=10, deadline=None)
@given(ep=st.sampled_from([1, 2]), rtp=st.sampled_from([1, 2]), moe_ep=st.sampled_from([1, 2]),
       fp8=st.booleans(), rrank=st.integers(0, 1))
def test_random_moe_layouts_cover_exactly(ep, rtp, moe_ep, fp8, rrank):
    arch = get_arch("tiny-qwen3-moe")
    if rtp % moe_ep:
        return
    megs = [dict(ep=ep, ep_rank=e) for e in range(ep)]
    sgl = dict(tp=rtp, tp_rank=rrank % rtp, moe_ep=moe_ep, quant="fp8_experts" if fp8 else None)
    if fp8 and (arch.moe_ffn // (rtp // moe_ep)) % 128:
        return
    dtype = torch.bfloat16
    rl, rp, rmeta, rviews = _sync(arch, megs, sgl, dtype)
    exp = rl.allocate(dtype=dtype, fill=True)
    for n in rp:
        a, b = rp[n], exp[n]
        if a.dtype == torch.float8_e4m3fn:
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        if "embed_tokens" in n or "lm_head" in n:
            rows = rl.padded_vocab // rl.tp
            valid = max(0, min(rows, arch.vocab - rl.tp_rank * rows))
            a, b = a[:valid], b[:valid]
        assert torch.equal(a, b), n


@settings(max_examples=15, deadline=None)
@given(model=st.sampled_from(["tiny-llama", "tiny-qwen2", "tiny-qwen3", "tiny-mixtral", "tiny-deepseek-v3"]),
       world=st.integers(1, 5), dim=st.sampled_from([0, 1]), rtp=st.sampled_from([1, 2]),
       rrank=st.integers(0, 1))
def test_random_fsdp_shardings_cover_exactly(model, world, dim, rtp, rrank):
    """FSDP trainers (any world size, rows or columns) into SGLang ranks: every bound element
    written once with the right value, vocab padding untouched."""
    from weightbridge_b200.parallel.fsdp import FSDPLayout
    arch = get_arch(model)
    senders, keep = [], []
    for i in range(world):
        lay = FSDPLayout(arch, world=world, rank=i, dim=dim)
        p = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(p)
        keep.append(p)
        senders.append(phys_binding(bind(meta, views)))
    rl = SGLangLayout(arch, tp=rtp, tp_rank=rrank % rtp, moe_ep=rtp if arch.is_moe else 1)
    rp = rl.allocate(dtype=torch.float32, pool=True)
    torch.empty(0, dtype=torch.uint8).set_(next(iter(rp.values())).untyped_storage()).fill_(0xFF)
    rmeta, rviews = rl.to_wb(rp)
    rphys = phys_binding(bind(rmeta, rviews))
    for sp in senders:
        cpu_execute(lower_ops(plan_pair(sp, rphys), ABS, ABS, item_bytes=4096))
    exp = rl.allocate(dtype=torch.float32, fill=True)
    for name, v in rviews.items():
        for t in v if isinstance(v, list) else [v]:
            assert not torch.isnan(t).any(), f"{name} not fully written"
    for n in rp:
        if "embed_tokens" in n or "lm_head" in n:
            valid = max(0, min(rl.padded_vocab // rl.tp, arch.vocab - rl.tp_rank * (rl.padded_vocab // rl.tp)))
            assert torch.equal(rp[n][:valid], exp[n][:valid])
            assert torch.isnan(rp[n][valid:]).all()
        else:
            assert torch.equal(rp[n], exp[n]), n


@settings(max_examples=20, deadline=None)
@given(mtp=st.sampled_from([1, 2, 4]), mpp=st.sampled_from([1, 3]), ep=st.sampled_from([1, 2]),
       etp=st.sampled_from([1, 2]), rtp=st.sampled_from([1, 2, 4]), attn_dp=st.booleans(),
       fp8=st.booleans(), rrank=st.integers(0, 3))
def test_random_mla_moe_layouts_cover_exactly(mtp, mpp, ep, etp, rtp, attn_dp, fp8, rrank):
    """DeepSeek-style layouts (MLA, dense first layer, shared experts, router bias) from random
    Megatron TP x PP x EP x ETP into a random SGLang rank, fp8 experts or not: every bound
    element (the derived w_kc / w_vc included) gets its value, vocab padding stays poisoned.
    Expert slices that cut fp8 blocks are quantised with the block amax merged over senders."""
    import numpy as np
    from weightbridge_b200.ops.executor import cpu_piece_amax
    arch = get_arch("tiny-deepseek-v3")
    sgl = dict(tp=rtp, tp_rank=rrank % rtp, moe_ep=rtp if fp8 else 1, quant="fp8_experts" if fp8 else None)
    if attn_dp:
        sgl.update(attn_tp=1, attn_tp_rank=0)
    rl = SGLangLayout(arch, **sgl)
    rp = rl.allocate(dtype=torch.bfloat16, pool=True)
    pool = torch.empty(0, dtype=torch.uint8).set_(next(iter(rp.values())).untyped_storage())
    pool.fill_(0xFF)                       # one allocation: poison it whole (w_kc / w_vc are transposed views)
    rmeta, rviews = rl.to_wb(rp)
    rphys = phys_binding(bind(rmeta, rviews))
    keep, tables = [], []
    for p in range(mpp):
        for e in range(ep):
            for t in range(max(mtp, etp)):
                lay = MegatronLayout(arch, tp=mtp, pp=mpp, ep=ep, etp=etp, tp_rank=t % mtp, pp_rank=p,
                                     ep_rank=e, etp_rank=t % etp)
                prm = lay.allocate(dtype=torch.bfloat16)
                keep.append(prm)
                tables.append(lower_ops(plan_pair(phys_binding(bind(*lay.to_wb(prm))), rphys), ABS, ABS,
                                        item_bytes=4096, receiver=0))
    block_amax = {}
    for tb in tables:                      # the senders' amax exchange, in one process
        for k, v in zip(tb.piece_keys, cpu_piece_amax(tb)):
            block_amax[k] = max(block_amax.get(k, 0.0), float(v))
    for tb in tables:
        cpu_execute(tb, np.array([block_amax[k] for k in tb.piece_keys], dtype=np.float32))
    exp = rl.allocate(dtype=torch.bfloat16, fill=True)
    for n in rp:
        a, b = rp[n], exp[n]
        if a.dtype == torch.float8_e4m3fn:
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        if "embed_tokens" in n or "lm_head" in n:
            rows = rl.padded_vocab // rl.tp
            valid = max(0, min(rows, arch.vocab - rl.tp_rank * rows))
            assert torch.isnan(rp[n][valid:]).all()
            a, b = a[:valid], b[:valid]
        assert torch.equal(a, b), n
