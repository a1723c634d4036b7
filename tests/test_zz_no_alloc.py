"""The no-allocation entry point ``wb_transfer_noalloc``, called through its exported C symbol.

It serves callers that cannot allocate GPU memory (an engine whose allocator already owns
the free memory, or a C host without a tensor framework): they pass the work table in host
memory and the library stages it into its fixed device scratch array.  These tests check that
it produces exactly what the regular entry point (``TransferProgram.launch``) produces, on
two calls in a row with different weights (the work table in pinned memory that the caller
overwrites as soon as each call returns), publishes the epoch to the flag, rejects tables
beyond its stated maximum without launching anything, and that calls after the first leave
the device's free memory and the caching allocator's counters unchanged.

The file is named so that pytest collects it last.
"""
import ctypes
import glob
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import weightbridge_b200
    pkg = os.path.dirname(weightbridge_b200.__file__)
    so = glob.glob(os.path.join(pkg, "_C*.so"))
    assert so, "native extension not built"
    lib = ctypes.CDLL(so[0])
    fn = lib.wb_transfer_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64,
                   ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _setup():
    from weightbridge_b200.core.binding import bind
    from weightbridge_b200.core.plan import Tables, lower_ops, phys_binding, plan_pair
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout

    dev = torch.device("cuda", 0)
    arch = get_arch("tiny-llama")
    senders = [MegatronLayout(arch, tp=2, tp_rank=r) for r in range(2)]
    sparams = [lay.allocate(device=dev, dtype=torch.bfloat16, seed=0) for lay in senders]
    rlay = SGLangLayout(arch, tp=1)
    outs = []
    for _ in range(2):      # receiver A: no-alloc entry point; receiver B: regular entry point
        rp = rlay.allocate(device=dev, dtype=torch.bfloat16)
        rmeta, rviews = rlay.to_wb(rp)
        rphys = phys_binding(bind(rmeta, rviews))
        parts = []
        for lay, sp in zip(senders, sparams):
            smeta, sviews = lay.to_wb(sp)
            parts.append(lower_ops(plan_pair(phys_binding(bind(smeta, sviews)), rphys), lambda a: 0, lambda a: 0,
                                   item_bytes=1 << 16))
        outs.append((rp, Tables.concat(parts)))
    return dev, senders, sparams, outs


def test_noalloc_entry_matches_regular_entry_on_two_calls():
    from weightbridge_b200.ops.executor import MODE_VECTOR, LaunchConfig, TransferProgram

    fn = _lib()
    dev, senders, sparams, ((rp_a, tab_a), (rp_b, tab_b)) = _setup()
    assert 0 < len(tab_a.items) <= 8192
    flag_a = torch.zeros(1, dtype=torch.int64, device=dev)
    flag_b = torch.zeros(1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    prog_b = TransferProgram(tab_b, dev, [flag_b.data_ptr()], LaunchConfig(mode=MODE_VECTOR))
    # the work table sits in pinned host memory and is overwritten (with empty items) as soon as
    # the call returns: the entry point must have taken its own copy by then
    table = np.ascontiguousarray(tab_a.items).view(np.uint8)
    pinned = torch.empty(table.nbytes, dtype=torch.uint8, pin_memory=True)
    items = pinned.numpy()
    flags = np.array([flag_a.data_ptr()], dtype=np.uint64)
    stream = torch.cuda.current_stream(dev)
    for call, seed in ((1, 11), (2, 12)):
        for lay, sp in zip(senders, sparams):
            lay.fill(sp, seed=seed)
        torch.cuda.synchronize()
        prog_b.launch(epoch=call)
        items[:] = table
        rc = fn(items.ctypes.data, len(tab_a.items), flags.ctypes.data, 1, call, status.data_ptr(),
                stream.cuda_stream)
        items[:] = 0
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and prog_b.read_status() == 0
        assert int(flag_a.item()) == call and int(flag_b.item()) == call
        for n in rp_a:
            assert torch.equal(rp_a[n], rp_b[n]), (call, n)
    # the second call delivered the second weights, not a leftover of the first
    from weightbridge_b200.parallel.sglang import SGLangLayout
    from weightbridge_b200.models.arch import get_arch
    exp = SGLangLayout(get_arch("tiny-llama"), tp=1).allocate(device=dev, dtype=torch.bfloat16, fill=True, seed=12)
    for n in rp_a:
        assert torch.equal(rp_a[n], exp[n]), n


def test_noalloc_rejects_oversized_tables():
    fn = _lib()
    big = np.zeros(8193 * 48, dtype=np.uint8)
    flags = np.zeros(65, dtype=np.uint64)
    stream = torch.cuda.current_stream(torch.device("cuda", 0))
    assert fn(big.ctypes.data, 8193, None, 0, 1, None, stream.cuda_stream) == -1
    assert fn(None, 0, flags.ctypes.data, 65, 1, None, stream.cuda_stream) == -2
    assert fn(None, 5, None, 0, 1, None, stream.cuda_stream) == -3
    torch.cuda.synchronize()


def test_noalloc_calls_allocate_no_device_memory():
    """After the first call on the device (which looks up the scratch array), further calls
    leave the device's free memory and the caching allocator's counters unchanged."""
    fn = _lib()
    dev, _senders, _sparams, ((_rp_a, tab_a), _b) = _setup()
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    items = np.ascontiguousarray(tab_a.items)
    flags = np.array([flag.data_ptr()], dtype=np.uint64)
    stream = torch.cuda.current_stream(dev)
    assert fn(items.ctypes.data, len(items), flags.ctypes.data, 1, 1, status.data_ptr(), stream.cuda_stream) == 0
    torch.cuda.synchronize()
    free0, _total = torch.cuda.mem_get_info(dev)
    keys = ("num_device_alloc", "num_device_free", "allocated_bytes.all.current", "reserved_bytes.all.current")
    stats0 = {k: torch.cuda.memory_stats(dev).get(k) for k in keys}
    for call in range(2, 7):
        rc = fn(items.ctypes.data, len(items), flags.ctypes.data, 1, call, status.data_ptr(), stream.cuda_stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
    assert int(flag.item()) == 6 and int(status.item()) == 0
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert {k: torch.cuda.memory_stats(dev).get(k) for k in keys} == stats0
