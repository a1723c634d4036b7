"""Microbenchmark of the transfer kernel on one GPU (also the small case for ncu captures).

  python -m weightbridge_b200.ops.microbench --case copy  --gbytes 1 --mode 1
  python -m weightbridge_b200.ops.microbench --case quant --gbytes 1
  python -m weightbridge_b200.ops.microbench --case strided --gbytes 1
  python -m weightbridge_b200.ops.microbench --case mc-peak --gbytes 2 --members 4   # >= 2 GPUs

copy:    one contiguous bf16 buffer -> another (HBM read + write), 16-byte aligned;
strided: column block of a row-major matrix -> contiguous (TP column split), 2-D items;
transpose: [heads, 128, 512] bf16 -> each matrix stored column-major (MLA's w_kc), OP_TRANSPOSE rows;
quant:   bf16 [E, 768, 2048] expert stack -> fp8 e4m3 + 128x128 fp32 block scales;
mixed:   half the bytes as the quant case, half as the copy case, in one program;
split:   the same stack as split-block pieces (half of every block: rows 64-127 of each block
         row), quantised by split_quant with an amax from split_amax (pass timed on the host);
peer-push / peer-pull / peer-quant (two GPUs, one process, peer access enabled): the kernel
         runs on GPU 0 and stores into GPU 1 (push), or runs on GPU 1 and loads from GPU 0
         (pull; plain and bulk loads from a peer, no cluster multicast), or quantises on
         GPU 0 into GPU 1; bandwidth counts the bytes that cross NVLink.
peer-peak: copy engine, push kernel and pull kernel GPU 0 -> GPU 1, best of --iters each;
         the largest is the measured peer peak (--out writes it as JSON).
Reports device time per launch (CUDA events, after warm-up) and achieved bandwidth against
the measured copy peak in MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..core.plan import Op, lower_ops
from .executor import LaunchConfig, TransferProgram


def _peak_gbs() -> float | None:
    here = os.path.dirname(os.path.abspath(__file__))
    p = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


PEER_PEAK_FILE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "profiles",
                              "nvlink_peer_peak.json")
MC_PEAK_FILE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "profiles",
                            "nvlink_multicast_store_peak.json")
FALLBACK_PEER_GBS = 770.0     # an earlier peer-copy measurement on B200s, used when no file exists


def _peer_peak_gbs() -> float:
    """The measured GPU -> GPU peak (largest of copy engine, push and pull kernels)."""
    try:
        return float(json.load(open(PEER_PEAK_FILE))["best_gbs"])
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEER_GBS


def _mc_peak_gbs() -> float | None:
    """The measured multicast store rate out of one GPU (``--case mc-peak``), if recorded."""
    try:
        return float(json.load(open(MC_PEAK_FILE))["best_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def build(case: str, gbytes: float, dev, item_bytes: int):
    n = int(gbytes * (1 << 30)) // 2
    if case == "copy":
        a = torch.randn(n, device=dev, dtype=torch.bfloat16)
        b = torch.empty_like(a)
        ops = [Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [n], [1], [1], a.dtype, a.dtype)]
        keep, traffic = (a, b), 2 * a.nbytes
    elif case == "strided":
        cols = 14336
        rows = max(1, n // cols)
        a = torch.randn(rows, cols, device=dev, dtype=torch.bfloat16)
        half = cols // 2
        b = torch.empty(rows, half, device=dev, dtype=torch.bfloat16)
        ops = [Op("copy", "x", (-1, a.data_ptr() + half * 2), (-1, b.data_ptr()), [rows, half], [cols, 1], [half, 1],
                  a.dtype, a.dtype)]
        keep, traffic = (a, b), 2 * b.nbytes
    elif case == "quant":
        r, c = 768, 2048
        e = max(1, n // (r * c))
        a = torch.randn(e, r, c, device=dev, dtype=torch.bfloat16)
        q = torch.empty(e, r, c, device=dev, dtype=torch.float8_e4m3fn)
        s = torch.empty(e, r // 128, c // 128, device=dev, dtype=torch.float32)
        ops = [Op("quant", "x", (-1, a[i].data_ptr()), (-1, q[i].data_ptr()), [r, c], [c, 1], [c, 1], a.dtype,
                  q.dtype, (-1, s[i].data_ptr()), [c // 128, 1], (128, 128)) for i in range(e)]
        keep, traffic = (a, q, s), a.nbytes + q.nbytes + s.nbytes
    elif case == "mixed":
        # one program of both kinds, as a Qwen3-MoE sync to an fp8-expert rollout: half the source
        # bytes are bf16 expert matrices quantised to e4m3, half a plain bf16 copy
        r, c = 768, 2048
        e = max(1, n // 2 // (r * c))
        a = torch.randn(e, r, c, device=dev, dtype=torch.bfloat16)
        q = torch.empty(e, r, c, device=dev, dtype=torch.float8_e4m3fn)
        s = torch.empty(e, r // 128, c // 128, device=dev, dtype=torch.float32)
        x = torch.randn(e * r * c, device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        ops = [Op("quant", "x", (-1, a[i].data_ptr()), (-1, q[i].data_ptr()), [r, c], [c, 1], [c, 1], a.dtype,
                  q.dtype, (-1, s[i].data_ptr()), [c // 128, 1], (128, 128)) for i in range(e)]
        ops.append(Op("copy", "y", (-1, x.data_ptr()), (-1, y.data_ptr()), [x.numel()], [1], [1], x.dtype, x.dtype))
        keep, traffic = (a, q, s, x, y), a.nbytes + q.nbytes + s.nbytes + 2 * x.nbytes
    elif case == "split":
        # expert-TP-like pieces: rows [64, 128) of every 128-row block row of a bf16 [E, 768, 2048]
        # stack (half of each block), one piece per 128 x 128 block, quantised with a given amax
        r, c = 768, 2048
        e = max(1, n // (r * c))
        a = torch.randn(e, r, c, device=dev, dtype=torch.bfloat16)
        q = torch.empty(e, r, c, device=dev, dtype=torch.float8_e4m3fn)
        s = torch.empty(e, r // 128, c // 128, device=dev, dtype=torch.float32)
        ops = []
        for i in range(e):
            for bi in range(r // 128):
                for bj in range(c // 128):
                    r0, c0 = bi * 128 + 64, bj * 128
                    ops.append(Op("squant", "x", (-1, a[i].data_ptr() + (r0 * c + c0) * 2),
                                  (-1, q[i].data_ptr() + r0 * c + c0), [64, 128], [c, 1], [c, 1], a.dtype, q.dtype,
                                  (-1, s[i, bi, bj].data_ptr()), [c // 128, 1], (128, 128), key=("x", i, bi, bj)))
        keep, traffic = (a, q, s), e * r * c                # half the source (2 B) and half the fp8 (1 B)
    elif case == "transpose":
        # MLA's w_kc from kv_b_proj: per head a [128, 512] bf16 matrix stored column-major
        r, c = 128, 512
        m = max(1, n // (r * c))
        a = torch.randn(m, r, c, device=dev, dtype=torch.bfloat16)
        b = torch.empty(m, c, r, device=dev, dtype=torch.bfloat16)
        bt = b.transpose(1, 2)                                    # logical [m, r, c]
        ops = [Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [m, r, c], list(a.stride()),
                  list(bt.stride()), a.dtype, a.dtype)]
        keep, traffic = (a, b), 2 * a.nbytes
    elif case in ("peer-push", "peer-pull", "peer-quant"):
        from ._ext import ext
        if torch.cuda.device_count() < 2:
            raise SystemExit("peer cases need two GPUs")
        d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
        for a_, b_ in ((0, 1), (1, 0)):
            with torch.cuda.device(a_):
                ext().enable_peer_access(b_)
        if case == "peer-quant":
            r, c = 768, 2048
            e = max(1, n // (r * c))
            a = torch.randn(e, r, c, device=d0, dtype=torch.bfloat16)
            q = torch.empty(e, r, c, device=d1, dtype=torch.float8_e4m3fn)
            s_ = torch.empty(e, r // 128, c // 128, device=d1, dtype=torch.float32)
            ops = [Op("quant", "x", (-1, a[i].data_ptr()), (-1, q[i].data_ptr()), [r, c], [c, 1], [c, 1], a.dtype,
                      q.dtype, (-1, s_[i].data_ptr()), [c // 128, 1], (128, 128)) for i in range(e)]
            keep, traffic = (a, q, s_), q.nbytes + s_.nbytes
        else:
            a = torch.randn(n, device=d0, dtype=torch.bfloat16)
            b = torch.empty(n, device=d1, dtype=torch.bfloat16)
            ops = [Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [n], [1], [1], a.dtype, a.dtype)]
            keep, traffic = (a, b), a.nbytes
    else:
        raise SystemExit(f"unknown case {case}")
    return lower_ops(ops, lambda x: 0, lambda x: 0, item_bytes=item_bytes), keep, traffic


def _time_ms(fn, iters: int, warmup: int, stream=None) -> float:
    """Best single-launch device time of ``fn`` over ``iters`` launches (CUDA events on the
    launching stream, after ``warmup`` launches)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


def peer_peak(gbytes: float, iters: int, warmup: int, item_bytes: int) -> dict:
    """GPU 0 -> GPU 1 bandwidth of the three ways bytes can cross NVLink here: the copy engine
    (a cross-device tensor copy: cudaMemcpyAsync between peers), this library's kernel storing
    into the peer (push, TMA bulk mode), and the kernel on GPU 1 loading from GPU 0 (pull).
    Best launch of ``iters`` each, CUDA events, clocks sampled during the timed region.  The
    largest figure is the peer-bandwidth denominator of the benchmark's roofline."""
    from ..utils.timing import ClockSampler
    from ._ext import ext
    if torch.cuda.device_count() < 2:
        raise SystemExit("peer-peak needs two GPUs")
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    for a_, b_ in ((0, 1), (1, 0)):
        with torch.cuda.device(a_):
            ext().enable_peer_access(b_)
    n = int(gbytes * (1 << 30)) // 2
    a = torch.randn(n, device=d0, dtype=torch.bfloat16)
    b = torch.empty(n, device=d1, dtype=torch.bfloat16)
    ops = [Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [n], [1], [1], a.dtype, a.dtype)]
    tables = lower_ops(ops, lambda x: 0, lambda x: 0, item_bytes=item_bytes)
    out = {"bytes": a.nbytes, "iters": iters, "warmup": warmup}
    with ClockSampler() as clk:
        with torch.cuda.device(d0):
            s0 = torch.cuda.current_stream(d0)
            out["copy_engine_ms"] = _time_ms(lambda: b.copy_(a, non_blocking=True), iters, warmup, s0)
            push = TransferProgram(tables, d0, [], LaunchConfig(mode=1))
            out["push_kernel_ms"] = _time_ms(lambda: push.launch(0, s0, signal=False), iters, warmup, s0)
            assert push.read_status() == 0
        with torch.cuda.device(d1):
            s1 = torch.cuda.current_stream(d1)
            pull = TransferProgram(tables, d1, [], LaunchConfig(mode=1))
            out["pull_kernel_ms"] = _time_ms(lambda: pull.launch(0, s1, signal=False), iters, warmup, s1)
            assert pull.read_status() == 0
    assert torch.equal(a.to(d1), b)
    for k in ("copy_engine", "push_kernel", "pull_kernel"):
        out[k + "_gbs"] = round(a.nbytes / (out[k + "_ms"] / 1e3) / 1e9, 1)
    out["best_gbs"] = max(out[k + "_gbs"] for k in ("copy_engine", "push_kernel", "pull_kernel"))
    out["clocks"] = clk.summary()
    out["device"] = torch.cuda.get_device_name(d0)
    return out


def mc_peak(gbytes: float, iters: int, warmup: int, item_bytes: int, members: int) -> dict:
    """NVLink multicast store bandwidth out of GPU 0: one multicast object backed by a VMM
    allocation on each of ``members`` GPUs (GPU 0 included), all in this process; the transfer
    kernel on GPU 0 copies a local buffer to the object's address with ``multimem.st`` (OP_COPY_MC
    items, vector mode), so every member receives the bytes once.  Best launch of ``iters``,
    CUDA events, clocks sampled.  Beside it, the same kernel pushing plain copies to each other
    member in turn (unicast fan-out).  Every member is verified.  The multicast figure is the
    roofline denominator of a sender's multicast egress in the benchmark.

    One process holds every member, so no process can exit while another's memory is bound;
    the object is unmapped and unbound before the process ends, failure or not."""
    from ..parallel.vmm import VmmPool
    from ..utils.timing import ClockSampler
    from ._ext import ext
    k = min(members, torch.cuda.device_count())
    if k < 2:
        raise SystemExit("mc-peak needs two GPUs")
    if not all(ext().multicast_supported(d) for d in range(k)):
        raise SystemExit("a GPU reports no NVLink multicast")
    d0 = torch.device("cuda", 0)
    for d in range(1, k):
        with torch.cuda.device(0):
            ext().enable_peer_access(d)
    want = int(gbytes * (1 << 30))
    pools = [VmmPool(want, d, tail_bytes=0) for d in range(k)]
    size = pools[0].size
    out = {"bytes": size, "members": k, "iters": iters, "warmup": warmup}
    h, bound, va = ext().mc_create(size, k), [], None
    try:
        for d in range(k):
            ext().mc_add_device(h, d)
        for d in range(k):
            ext().mc_bind_mem(h, 0, pools[d].handle, 0, size)
            bound.append(d)
        va = ext().mc_map(h, size, 0)[0]
        n = size // 2
        a = torch.randn(n, device=d0, dtype=torch.bfloat16)
        ops = [Op("copy", "x", (-1, a.data_ptr()), (-1, 0), [n], [1], [1], a.dtype, a.dtype)]
        mc_tables = lower_ops(ops, lambda x: 0, lambda x: va, item_bytes=item_bytes, multicast=True)
        # unicast comparison: plain peer tensors (caching allocator, peer access enabled above);
        # the members' VMM pools are mapped for their own GPU only, so GPU 0 must not store there
        peers = [torch.empty(n, device=torch.device("cuda", d), dtype=torch.bfloat16) for d in range(1, k)]
        uc_tables = lower_ops([Op("copy", "x", (-1, a.data_ptr()), (-1, b.data_ptr()), [n], [1], [1], a.dtype, a.dtype)
                               for b in peers], lambda x: 0, lambda x: 0, item_bytes=item_bytes)
        with ClockSampler() as clk, torch.cuda.device(d0):
            s0 = torch.cuda.current_stream(d0)
            mc = TransferProgram(mc_tables, d0, [], LaunchConfig(mode=0))
            out["multicast_ms"] = _time_ms(lambda: mc.launch(0, s0, signal=False), iters, warmup, s0)
            assert mc.read_status() == 0, mc.read_status()
            torch.cuda.synchronize()
            ok = [torch.equal(pools[d].tensor[: a.nbytes].view(torch.bfloat16).to(d0), a) for d in range(k)]
            uc = TransferProgram(uc_tables, d0, [], LaunchConfig(mode=1))
            out["unicast_fanout_ms"] = _time_ms(lambda: uc.launch(0, s0, signal=False), iters, warmup, s0)
            assert uc.read_status() == 0, uc.read_status()
        out["verified_members"] = ok
        out["multicast_egress_gbs"] = round(a.nbytes / (out["multicast_ms"] / 1e3) / 1e9, 1)
        out["unicast_fanout_egress_gbs"] = round(a.nbytes * (k - 1) / (out["unicast_fanout_ms"] / 1e3) / 1e9, 1)
        out["best_gbs"] = out["multicast_egress_gbs"]
        out["clocks"] = clk.summary()
        out["device"] = torch.cuda.get_device_name(d0)
        ok += [torch.equal(b.to(d0), a) for b in peers]
        out["verified_members"] = ok
        del mc, uc, a, peers
        torch.cuda.synchronize()
    finally:
        if va is not None:
            ext().va_unmap(va, size)
        for d in bound:
            ext().mc_unbind(h, d, 0, size)
        ext().mem_release(h)
        for p_ in pools:
            p_.free()
    if not all(out.get("verified_members", [False])):
        raise SystemExit(f"multicast copy mismatch: {out}")
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--case", default="copy",
                   choices=["copy", "strided", "transpose", "quant", "mixed", "split", "peer-push", "peer-pull", "peer-quant",
                            "peer-peak", "mc-peak"])
    p.add_argument("--gbytes", type=float, default=1.0)
    p.add_argument("--mode", type=int, default=-1)
    p.add_argument("--piece", type=int, default=16384)
    p.add_argument("--grid", type=int, default=0)
    p.add_argument("--item-bytes", type=int, default=1 << 19)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--out", default=None, help="peer-peak, mc-peak: also write the JSON result to this file")
    p.add_argument("--members", type=int, default=4, help="mc-peak: GPUs in the multicast object")
    a = p.parse_args(argv)
    if a.case == "mc-peak":
        res = mc_peak(a.gbytes, a.iters, a.warmup, a.item_bytes, a.members)
        print(json.dumps(res))
        if a.out:
            with open(a.out, "w") as f:
                json.dump(res, f, indent=1)
        return
    if a.case == "peer-peak":
        res = peer_peak(a.gbytes, a.iters, a.warmup, a.item_bytes)
        print(json.dumps(res))
        if a.out:
            with open(a.out, "w") as f:
                json.dump(res, f, indent=1)
        return
    dev = torch.device("cuda", 1 if a.case == "peer-pull" else 0)   # pull: the kernel runs on the reader
    torch.cuda.set_device(dev)
    tables, keep, traffic = build(a.case, a.gbytes, dev, a.item_bytes)
    prog = TransferProgram(tables, dev, [], LaunchConfig(mode=a.mode, piece_bytes=a.piece, grid=a.grid or None))
    if prog.n_pieces:          # split pieces: a real amax pass first, timed separately
        import numpy as np
        import time
        t0 = time.perf_counter()
        part = prog.piece_amax()
        amax_ms = (time.perf_counter() - t0) * 1e3
        prog.set_piece_amax(np.asarray(part, dtype=np.float32))
    for _ in range(a.warmup):
        prog.launch(0, signal=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        prog.launch(0, signal=False)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    gbs = traffic / (ms / 1e3) / 1e9
    peak = _peer_peak_gbs() if a.case.startswith("peer") else _peak_gbs()   # measured peer vs HBM copy
    print(json.dumps({"case": a.case, "gbytes": a.gbytes, "mode": prog.config.mode, "launch_mode": prog.launch_mode,
                      "tma_quant_blocks": prog.n_tma_quant, "piece": a.piece, "grid": prog.grid(),
                      "items": len(tables.items), "qwork": len(tables.qwork), "pieces": len(tables.pieces),
                      "amax_pass_ms_host": round(amax_ms, 3) if prog.n_pieces else None, "ms": round(ms, 4),
                      "traffic_bytes": traffic, "gbs": round(gbs, 1),
                      "frac_of_measured": round(gbs / peak, 3) if peak else None,
                      "status": prog.read_status()}))


if __name__ == "__main__":
    main()
