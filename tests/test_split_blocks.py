"""fp8 blocks split across senders (core/splitq.py): geometry of the split, the amax
exchange, the host kernels against the whole-tensor oracle, and the full protocol over gloo."""
import numpy as np
import pytest
import torch
from hypothesis import given, settings, strategies as st

from weightbridge_b200.core.plan import lower_ops, plan_pair, validate_tables, storage_ranges
from weightbridge_b200.core.splitq import AmaxExchange, block_split, split_keys
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.ops.executor import cpu_execute, cpu_piece_amax
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout
from tests.test_plan_cpu import ABS, make_receiver, make_senders, _u8


def test_block_split_aligned_region_is_all_core():
    core, pieces = block_split([(128, 384, 768), (0, 256, 256)], (128, 128))
    assert core == ((128, 384), (0, 256)) and pieces == []


def test_block_split_expert_tp_slice():
    # rows [192, 384) of 768: block row 1 ([128, 256)) is shared, block rows 2 is whole
    core, pieces = block_split([(192, 384, 768), (0, 256, 256)], (128, 128))
    assert core == ((256, 384), (0, 256))
    assert pieces == [((1, 0), (192, 256), (0, 128)), ((1, 1), (192, 256), (128, 256))]


def test_block_split_partial_last_block_at_tensor_end_is_whole():
    core, pieces = block_split([(128, 200, 200), (0, 100, 100)], (128, 128))
    assert core == ((128, 200), (0, 100)) and pieces == []


def test_block_split_inside_one_block():
    core, pieces = block_split([(10, 20, 256), (30, 40, 256)], (128, 128))
    assert core is None and pieces == [((0, 0), (10, 20), (30, 40))]


@settings(max_examples=300, deadline=None)
@given(st.integers(1, 700), st.integers(1, 700), st.data())
def test_block_split_partitions_the_region(wr, wc, data):
    r0 = data.draw(st.integers(0, wr - 1))
    r1 = data.draw(st.integers(r0 + 1, wr))
    c0 = data.draw(st.integers(0, wc - 1))
    c1 = data.draw(st.integers(c0 + 1, wc))
    bn, bk = data.draw(st.sampled_from([(128, 128), (64, 32), (16, 128)]))
    core, pieces = block_split([(r0, r1, wr), (c0, c1, wc)], (bn, bk))
    cover = np.zeros((wr, wc), dtype=np.int32)
    if core is not None:
        (a, b), (c, d) = core
        assert a % bn == 0 and c % bk == 0
        assert (b % bn == 0 or b == wr) and (d % bk == 0 or d == wc)
        cover[a:b, c:d] += 1
    for (bi, bj), (a, b), (c, d) in pieces:
        assert bi * bn <= a < b <= min((bi + 1) * bn, wr) and bj * bk <= c < d <= min((bj + 1) * bk, wc)
        # a piece never covers its whole block
        assert (a, b, c, d) != (bi * bn, min((bi + 1) * bn, wr), bj * bk, min((bj + 1) * bk, wc))
        cover[a:b, c:d] += 1
    expect = np.zeros_like(cover)
    expect[r0:r1, c0:c1] = 1
    assert np.array_equal(cover, expect)


def test_exchange_merges_common_blocks_only():
    keys = {0: [(4, "w", 0, 0), (4, "w", 1, 0)], 1: [(4, "w", 1, 0), (4, "w", 2, 0)], 2: [(5, "w", 0, 0)]}
    x = AmaxExchange(0, keys)
    assert x.co_owners == [1]
    pos = x.positions([(4, "w", 1, 0), (4, "w", 0, 0), (4, "w", 1, 0)])
    vals = x.local(np.array([1.0, 5.0, 3.0], np.float32), pos)
    assert vals.tolist() == [5.0, 3.0]
    merged = x.merge(vals, {1: np.array([7.0, 9.0], np.float32)})
    assert merged.tolist() == [5.0, 7.0]
    with pytest.raises(ValueError):
        x.merge(vals, {1: np.array([7.0], np.float32)})


@pytest.mark.parametrize("etp", [4, 8])
def test_split_blocks_host_kernels_match_whole_tensor_oracle(etp):
    """Expert TP slices of 64 / 32 rows cut every 128 x 128 block of the experts: each
    sender's pieces, quantised with the block amax merged over all senders, reproduce the
    oracle's quantisation of the whole tensor bit for bit."""
    arch = get_arch("tiny-qwen3-moe")
    senders = make_senders([MegatronLayout(arch, etp=etp, etp_rank=i) for i in range(etp)], torch.bfloat16)
    lay = SGLangLayout(arch, tp=1, quant="fp8_experts")
    params, rmeta, rphys = make_receiver(lay, torch.bfloat16)
    tables, partials = [], []
    for p, smeta, sphys in senders:
        t = lower_ops(plan_pair(sphys, rphys), ABS, ABS, receiver=0)
        assert len(t.pieces) and len(t.qwork) == 0          # every expert block is split
        validate_tables(t, storage_ranges(p.values()), storage_ranges(params.values()))
        assert sorted(set(k[1:] for k in t.piece_keys)) == split_keys(smeta, rmeta)
        tables.append(t)
        partials.append(cpu_piece_amax(t))
    block_amax: dict = {}
    for t, part in zip(tables, partials):
        for k, a in zip(t.piece_keys, part):
            block_amax[k] = max(block_amax.get(k, 0.0), float(a))
    for t in tables:
        cpu_execute(t, np.array([block_amax[k] for k in t.piece_keys], dtype=np.float32))
    expected = lay.allocate(dtype=torch.bfloat16, fill=True)
    for n in params:
        assert torch.equal(_u8(params[n]), _u8(expected[n])), n


def test_split_pieces_refuse_to_run_without_block_amax():
    arch = get_arch("tiny-qwen3-moe")
    (_p, _m, sphys), = make_senders([MegatronLayout(arch, etp=4, etp_rank=1)], torch.bfloat16)
    _params, _rm, rphys = make_receiver(SGLangLayout(arch, tp=1, quant="fp8_experts"), torch.bfloat16)
    with pytest.raises(ValueError, match="block amax"):
        cpu_execute(lower_ops(plan_pair(sphys, rphys), ABS, ABS))


def test_split_blocks_expert_tp4_to_tp1_fp8_gloo():
    """Four trainer ranks with expert TP 4 (64-row slices of the experts), one fp8 rollout
    worker: the senders exchange the amax of every shared block through the session."""
    from tests.e2e_harness import run
    run("tiny-qwen3-moe", "cpu_direct", [dict(etp=4, etp_rank=i) for i in range(4)],
        dict(tp=1, quant="fp8_experts"), dtype=torch.bfloat16, n_syncs=2)


@settings(max_examples=12, deadline=None)
@given(world=st.integers(1, 7), tp=st.sampled_from([1, 2]), dim=st.sampled_from([0, 1]),
       f32=st.booleans())
def test_split_blocks_random_fsdp_shardings(world, tp, dim, f32):
    """Random FSDP-style shardings (any world size, rows or columns) into fp8 SGLang ranks:
    whole blocks, split blocks and their exchange reproduce the oracle bit for bit."""
    from weightbridge_b200.parallel.fsdp import FSDPLayout
    dtype = torch.float32 if f32 else torch.bfloat16
    arch = get_arch("tiny-llama-fp8")
    senders = make_senders([FSDPLayout(arch, world=world, rank=i, dim=dim) for i in range(world)], dtype)
    for r in range(tp):
        lay = SGLangLayout(arch, tp=tp, tp_rank=r, quant="fp8_linear")
        params, _rmeta, rphys = make_receiver(lay, dtype)
        tables = [lower_ops(plan_pair(sphys, rphys), ABS, ABS, receiver=r) for _p, _m, sphys in senders]
        block: dict = {}
        for t in tables:
            for k, a in zip(t.piece_keys, cpu_piece_amax(t)):
                block[k] = max(block.get(k, 0.0), float(a))
        for t in tables:
            cpu_execute(t, np.array([block[k] for k in t.piece_keys], dtype=np.float32))
        expected = lay.allocate(dtype=dtype, fill=True)
        for n in params:
            assert torch.equal(_u8(params[n]), _u8(expected[n])), (n, world, tp, dim)


@settings(max_examples=12, deadline=None)
@given(model=st.sampled_from(["tiny-llama-fp8", "tiny-qwen2-moe"]), mtp=st.sampled_from([1, 2]),
       mpp=st.sampled_from([1, 2]), rtp=st.sampled_from([1, 2]), f32=st.booleans())
def test_random_megatron_to_fp8_linear(model, mtp, mpp, rtp, f32):
    """Random Megatron TP x PP layouts into fp8 SGLang ranks (every linear layer quantised):
    grouped-QKV regions cut per KV group, blocks split between ranks merged by amax."""
    dtype = torch.float32 if f32 else torch.bfloat16
    arch = get_arch(model)
    if arch.num_kv_heads % mtp:
        return
    megs = [MegatronLayout(arch, tp=mtp, pp=mpp, tp_rank=t, pp_rank=p) for t in range(mtp) for p in range(mpp)]
    senders = make_senders(megs, dtype)
    for r in range(rtp):
        try:
            lay = SGLangLayout(arch, tp=rtp, tp_rank=r, quant="fp8_linear", moe_ep=rtp if arch.is_moe else 1)
            params, _rmeta, rphys = make_receiver(lay, dtype)
        except ValueError:            # a TP split the fp8 layout itself refuses (block-misaligned)
            return
        tables = [lower_ops(plan_pair(sphys, rphys), ABS, ABS, receiver=r) for _p, _m, sphys in senders]
        block: dict = {}
        for t in tables:
            for k, a in zip(t.piece_keys, cpu_piece_amax(t)):
                block[k] = max(block.get(k, 0.0), float(a))
        for t in tables:
            cpu_execute(t, np.array([block[k] for k in t.piece_keys], dtype=np.float32))
        expected = lay.allocate(dtype=dtype, fill=True)
        for n in params:
            assert torch.equal(_u8(params[n]), _u8(expected[n])), (n, model, mtp, mpp, rtp)
