"""sm_100a transfer kernel on one GPU: every mode against the C++ CPU executor / torch oracle.

Numerics: copies and casts must be bit-exact against the CPU executor; fp8 block
quantisation bit-exact against the plain-PyTorch fp32 reference (``quant_ref``).  Bounded
waits are exercised with a flag that nothing sets: the kernel must return with
ST_FLAG_TIMEOUT, and the context must stay usable.
"""
import random
import time

import pytest
import torch

from weightbridge_b200.core.binding import bind
from weightbridge_b200.core.plan import Op, lower_ops, phys_binding, plan_pair
from weightbridge_b200.core.shard import box_copy, coalesce
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.ops._ext import ext
from weightbridge_b200.ops.executor import (MODE_BULK4, MODE_BULK8, MODE_BULK12, MODE_VECTOR, LaunchConfig,
                                            TransferProgram, cpu_execute, wait_flags)
from weightbridge_b200.ops.quant_ref import block_quant_fp8_ref
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout

pytestmark = pytest.mark.gpu
ABS = lambda _a: 0
MODES = [MODE_VECTOR, MODE_BULK8, MODE_BULK12, MODE_BULK4]


def _u8(t):
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


def _sync(meg, sgl, dtype, mode, item_bytes=1 << 19, piece=16384):
    dev = torch.device("cuda", 0)
    senders = []
    for lay in meg:
        params = lay.allocate(device=dev, dtype=dtype)
        meta, views = lay.to_wb(params)
        senders.append((params, phys_binding(bind(meta, views))))
    out = []
    for lay in sgl:
        params = lay.allocate(device=dev, dtype=dtype)
        meta, views = lay.to_wb(params)
        rphys = phys_binding(bind(meta, views))
        flag = torch.zeros(1, dtype=torch.int64, device=dev)
        for _p, sphys in senders:
            t = lower_ops(plan_pair(sphys, rphys), ABS, ABS, item_bytes=item_bytes)
            prog = TransferProgram(t, dev, [flag.data_ptr()], LaunchConfig(mode=mode, piece_bytes=piece))
            prog.launch(epoch=3)
            torch.cuda.synchronize()
            assert prog.read_status() == 0
            assert int(flag.item()) == 3
            flag.zero_()
        out.append((lay, params))
    return out


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("model,meg,sgl", [
    ("tiny-llama", [dict(tp=2, tp_rank=i) for i in range(2)], [dict(tp=4, tp_rank=i) for i in range(4)]),
    ("tiny-qwen2", [dict(pp=2, pp_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i) for i in range(2)]),
    ("tiny-qwen3-moe", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i) for i in range(2)]),
])
def test_gpu_layout_sync_bitwise(mode, model, meg, sgl):
    arch = get_arch(model)
    res = _sync([MegatronLayout(arch, **m) for m in meg], [SGLangLayout(arch, **s) for s in sgl],
                torch.bfloat16, mode, item_bytes=8192)
    for lay, params in res:
        expected = lay.allocate(device="cuda", dtype=torch.bfloat16, fill=True)
        for n in params:
            assert torch.equal(params[n], expected[n]), n


@pytest.mark.parametrize("mode", MODES)
def test_gpu_fp8_expert_quant_matches_oracle(mode):
    arch = get_arch("tiny-qwen3-moe")
    meg = [MegatronLayout(arch, ep=2, ep_rank=i) for i in range(2)]
    sgl = [SGLangLayout(arch, tp=2, tp_rank=i, moe_ep=2, quant="fp8_experts") for i in range(2)]
    for lay, params in _sync(meg, sgl, torch.bfloat16, mode):
        expected = lay.allocate(device="cuda", dtype=torch.bfloat16, fill=True)
        for n in params:
            assert torch.equal(_u8(params[n]), _u8(expected[n])), n


def _quant_op(x, q, s):
    n, k = x.shape
    return Op("quant", "x", (-1, x.data_ptr()), (-1, q.data_ptr()), [n, k], [x.stride(0), 1], [q.stride(0), 1],
              x.dtype, torch.float8_e4m3fn, (-1, s.data_ptr()), [s.stride(0), 1], (128, 128))


def _quant_case(dev, src_dtype, n, k, seed=0, dst_pitch=None):
    """A random [n, k] source and its e4m3 destination (rows ``dst_pitch`` bytes apart) + scales."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(n, k, generator=g) * 3).to(src_dtype).to(dev)
    q = torch.zeros(n, dst_pitch or k, dtype=torch.float8_e4m3fn, device=dev)[:, :k]
    s = torch.zeros((n + 127) // 128, (k + 127) // 128, dtype=torch.float32, device=dev)
    return x, q, s


def _check_quant(x, q, s):
    qr, sr = block_quant_fp8_ref(x.cpu())
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(q.cpu().view(torch.uint8), qr.view(torch.uint8))


@pytest.mark.parametrize("mode", [MODE_VECTOR, MODE_BULK8, MODE_BULK4, MODE_BULK12])
def test_gpu_quant_partial_blocks_and_fp32_source(mode):
    """Edge blocks (rows/cols not multiples of 128), fp16 and fp32 sources, in every mode: in the
    TMA modes bf16/fp16 matrices whose columns are a multiple of 8 arrive by tensor-map loads
    (past-the-edge rows and columns read as zero), the others take the register path."""
    dev = torch.device("cuda", 0)
    # (dtype, shape, TMA-eligible, destination row pitch): 16-byte destination rows take the
    # 16-byte stores (also with a last block 8 columns wide), others 8-byte stores
    cases = [(torch.float32, (200, 300), False, None), (torch.bfloat16, (130, 256), True, None),
             (torch.float16, (64, 100), False, None), (torch.bfloat16, (257, 136), True, None),
             (torch.float16, (128, 384), True, None), (torch.bfloat16, (200, 264), True, 272)]
    for src_dtype, (n, k), tma, pitch in cases:
        x, q, s = _quant_case(dev, src_dtype, n, k, dst_pitch=pitch)
        prog = TransferProgram(lower_ops([_quant_op(x, q, s)], ABS, ABS), dev, [], LaunchConfig(mode=mode))
        nblocks = s.numel()
        assert prog.n_tma_quant == (nblocks if tma and mode != MODE_VECTOR else 0), (src_dtype, n, k)
        prog.launch(1)
        torch.cuda.synchronize()
        assert prog.read_status() == 0
        _check_quant(x, q, s)
        if pitch:                      # the row padding past column k stays untouched
            full = torch.as_strided(q, (n, pitch), (pitch, 1))
            assert not full[:, k:].view(torch.uint8).any()


@pytest.mark.parametrize("mode", [MODE_BULK8, MODE_BULK4])
def test_gpu_tma_quant_ring_wraps_and_mixes_with_register_blocks(mode):
    """Two CTAs walk 128 TMA blocks each (the shared-memory ring of 2-4 stages wraps many times,
    mbarrier parities flip) interleaved with register-path blocks of a matrix whose rows start
    2 bytes off a 16-byte boundary, and with plain copies; three launches in a row."""
    dev = torch.device("cuda", 0)
    a, qa, sa = _quant_case(dev, torch.bfloat16, 1024, 4096, seed=1)          # 256 TMA blocks
    buf = torch.zeros(300 * 257 + 1, dtype=torch.bfloat16, device=dev)
    b = buf[1:].view(300, 257)[:, :256]                                         # misaligned rows: register path
    b.copy_((torch.randn(300, 256) * 0.5).to(torch.bfloat16))
    qb = torch.zeros(300, 256, dtype=torch.float8_e4m3fn, device=dev)
    sb = torch.zeros(3, 2, dtype=torch.float32, device=dev)
    c = torch.randn(4096, device=dev)
    d = torch.zeros_like(c)
    ops = [_quant_op(a, qa, sa), _quant_op(b, qb, sb),
           Op("copy", "c", (-1, c.data_ptr()), (-1, d.data_ptr()), [4096], [1], [1], c.dtype, c.dtype)]
    prog = TransferProgram(lower_ops(ops, ABS, ABS), dev, [], LaunchConfig(mode=mode, grid=2))
    assert prog.n_tma_quant == 256 and prog.launch_mode == mode
    for ep in range(1, 4):
        qa.zero_(); sa.zero_(); qb.zero_(); sb.zero_(); d.zero_()
        prog.launch(ep)
        torch.cuda.synchronize()
        assert prog.read_status() == 0
        _check_quant(a, qa, sa)
        _check_quant(b, qb, sb)
        assert torch.equal(c, d)


def _random_ops(rng, dev, count=12):
    """Random strided copies of odd sizes/offsets (exercise 1/2/4/8/16-byte paths)."""
    ops, pairs = [], []
    for _ in range(count):
        dtype = rng.choice([torch.uint8, torch.float16, torch.float32, torch.bfloat16])
        shape = [rng.randint(1, 40), rng.randint(1, 70)]
        a = torch.randint(0, 100, shape, device=dev).to(dtype)
        b = torch.zeros(shape, dtype=dtype, device=dev)
        r0, c0 = rng.randrange(shape[0]), rng.randrange(shape[1])
        r1, c1 = rng.randint(r0 + 1, shape[0]), rng.randint(c0 + 1, shape[1])
        box = [(r0, r1, shape[0]), (c0, c1, shape[1])]
        full = [(0, shape[0], shape[0]), (0, shape[1], shape[1])]
        bc = box_copy(full, box, list(a.stride()), [shape[1], 1])
        e, ss, ds = coalesce(bc.extents, bc.src_strides, bc.dst_strides)
        es = a.element_size()
        ops.append(Op("copy", "x", (-1, a.data_ptr() + bc.src_offset * es),
                      (-1, b.data_ptr() + (r0 * shape[1] + c0) * es), e, ss, ds, dtype, dtype))
        pairs.append((a, b, box))
    return ops, pairs


@pytest.mark.parametrize("mode", MODES)
def test_gpu_random_strided_copies(mode):
    rng = random.Random(mode)
    dev = torch.device("cuda", 0)
    ops, pairs = _random_ops(rng, dev)
    prog = TransferProgram(lower_ops(ops, ABS, ABS, item_bytes=512), dev, [], LaunchConfig(mode=mode, piece_bytes=256))
    prog.launch(1)
    torch.cuda.synchronize()
    assert prog.read_status() == 0
    for a, b, box in pairs:
        sl = tuple(slice(l, r) for l, r, _ in box)
        assert torch.equal(b[sl], a[sl])
        mask = torch.ones_like(b, dtype=torch.bool)
        mask[sl] = False
        assert not b[mask].any()


def test_gpu_matches_cpu_executor_on_cast():
    dev = torch.device("cuda", 0)
    x = torch.randn(333, 77, device=dev)
    for dst_dtype in (torch.bfloat16, torch.float16):
        y = torch.zeros(333, 77, dtype=dst_dtype, device=dev)
        op = Op("cast", "x", (-1, x.data_ptr()), (-1, y.data_ptr()), [333 * 77], [1], [1], torch.float32, dst_dtype)
        prog = TransferProgram(lower_ops([op], ABS, ABS, item_bytes=4096), dev, [], LaunchConfig(mode=MODE_VECTOR))
        prog.launch(1)
        torch.cuda.synchronize()
        xc = x.cpu()
        yc = torch.zeros(333, 77, dtype=dst_dtype)
        opc = Op("cast", "x", (-1, xc.data_ptr()), (-1, yc.data_ptr()), [333 * 77], [1], [1], torch.float32, dst_dtype)
        cpu_execute(lower_ops([opc], ABS, ABS))
        assert torch.equal(y.cpu(), yc)
        assert torch.equal(yc, xc.to(dst_dtype))


def test_wait_flags_times_out_with_status():
    dev = torch.device("cuda", 0)
    flags = torch.zeros(3, dtype=torch.int64, device=dev)
    epoch = torch.tensor([5], dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    where = torch.full((1,), 0x7FFFFFFF, dtype=torch.int32, device=dev)
    t0 = time.time()
    wait_flags(flags, epoch, 0.05, status, where)
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert int(status.item()) & ext().ST_FLAG_TIMEOUT
    assert int(where.item()) == 0
    # the context is still usable, and a satisfied wait reports nothing
    flags.fill_(5)
    status.zero_()
    wait_flags(flags, epoch, 0.05, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    flags[1] = 9
    wait_flags(flags, epoch, 0.05, status)
    torch.cuda.synchronize()
    assert int(status.item()) & ext().ST_FLAG_STALE


def test_repeated_launches_reset_counter():
    dev = torch.device("cuda", 0)
    a = torch.randn(1 << 20, device=dev)
    b = torch.zeros_like(a)
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    op = Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [a.numel()], [1], [1], a.dtype, a.dtype)
    prog = TransferProgram(lower_ops([op], ABS, ABS, item_bytes=1 << 16), dev, [flag.data_ptr()],
                           LaunchConfig(mode=MODE_BULK8))
    for e in range(1, 6):
        prog.launch(e)
        torch.cuda.synchronize()
        assert int(flag.item()) == e
        assert int(prog.counter.item()) == 0
    assert torch.equal(a, b)


@pytest.mark.parametrize("etp,dtype", [(4, torch.bfloat16), (8, torch.bfloat16), (4, torch.float32)])
def test_gpu_split_blocks_match_whole_tensor_oracle(etp, dtype):
    """fp8 blocks split across senders (expert TP slices of 64 / 32 rows): split_amax on every
    sender's pieces, the block amax merged over the senders on the host, split_quant plus the
    transfer kernel; the receiver equals the oracle's quantisation of the whole tensor.  The
    down_proj pieces (64 / 32 columns) take the element path, gate/up pieces with bf16 sources
    the vector path."""
    import numpy as np
    dev = torch.device("cuda", 0)
    arch = get_arch("tiny-qwen3-moe")
    lay = SGLangLayout(arch, tp=1, quant="fp8_experts")
    rparams = lay.allocate(device=dev, dtype=dtype)
    rmeta, rviews = lay.to_wb(rparams)
    rphys = phys_binding(bind(rmeta, rviews))
    progs, keep = [], []
    for i in range(etp):
        meg = MegatronLayout(arch, etp=etp, etp_rank=i)
        sp = meg.allocate(device=dev, dtype=dtype)
        keep.append(sp)
        smeta, sviews = meg.to_wb(sp)
        t = lower_ops(plan_pair(phys_binding(bind(smeta, sviews)), rphys), ABS, ABS, receiver=0)
        assert len(t.pieces)
        progs.append(TransferProgram(t, dev, [], LaunchConfig(mode=MODE_VECTOR)))
    block = {}
    partials = [p.piece_amax() for p in progs]
    for p, part in zip(progs, partials):
        for k, a in zip(p.tables.piece_keys, part):
            block[k] = max(block.get(k, 0.0), float(a))
    for p in progs:
        p.set_piece_amax(np.array([block[k] for k in p.tables.piece_keys], dtype=np.float32))
        p.launch(epoch=1, signal=False)
    torch.cuda.synchronize()
    assert all(p.read_status() == 0 for p in progs)
    expected = lay.allocate(device=dev, dtype=dtype, fill=True)
    for n in rparams:
        assert torch.equal(_u8(rparams[n]), _u8(expected[n])), n


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_gpu_synth_fill_kernel_matches_torch_ops(dtype):
    """The native fill kernel writes, into strided views, exactly the values the torch-op
    statement of the same arithmetic produces on the GPU (boxes with offsets, 1-D to 3-D)."""
    from weightbridge_b200.models.synthetic import synth_fill, synth_values
    dev = torch.device("cuda", 0)
    full = torch.zeros(96, 3 * 160, dtype=dtype, device=dev)
    cases = [
        ("w.col", full[:, 160:320], [(32, 128, 512), (160, 320, 480)]),          # column block, row offset
        ("w.grp", full[:, :150].unflatten(1, (3, 50)), [(0, 96, 96), (1, 4, 7), (5, 55, 60)]),
        ("w.flat", torch.zeros(4099, dtype=dtype, device=dev)[3:], [((1 << 33) + 5, (1 << 33) + 4101, 1 << 40)]),
    ]
    for name, view, box in cases:
        synth_fill(view, name, box, seed=3)
        ref = synth_values(name, box, dev, dtype, seed=3)
        assert torch.equal(view.contiguous().view(torch.uint8 if dtype != torch.float32 else torch.int32),
                           ref.contiguous().view(torch.uint8 if dtype != torch.float32 else torch.int32)), name


@pytest.mark.parametrize("mode", [MODE_VECTOR, MODE_BULK8])
@pytest.mark.parametrize("dtype,offs", [(torch.bfloat16, (0, 0)), (torch.bfloat16, (1, 3)), (torch.float32, (1, 0)),
                                        (torch.uint8, (0, 5))])
def test_gpu_transposed_destination(mode, dtype, offs):
    """OP_TRANSPOSE work rows (a destination stored column-major, like MLA's w_kc): the
    2-byte tile path (aligned and misaligned rows, edge tiles) and the element path write
    exactly the transpose, in every kernel mode; nothing outside the destination changes."""
    from tests.test_plan_cpu import _transpose_case
    dev = torch.device("cuda", 0)
    op, src, dst, store, es = _transpose_case(dtype, 3, 70, 130, src_off=offs[0], dst_off=offs[1], device=dev)
    prog = TransferProgram(lower_ops([op], ABS, ABS, item_bytes=64 * 70 * es), dev, [], LaunchConfig(mode=mode))
    prog.launch(1)
    torch.cuda.synchronize()
    assert prog.read_status() == 0
    assert torch.equal(dst, src)
    assert not store[:offs[1]].to(torch.float32).any()
