"""Environment check for a weight-sync deployment: ``python -m weightbridge_b200.doctor``.

Prints one JSON object: the native extension (and the file it was loaded from), torch / CUDA /
NCCL versions, and per GPU its name, compute capability, SM count and multicast (NVLS)
support, plus the peer-access matrix that ``gpu_direct`` relies on and the measured NVLink
figures the planner's estimates use (``profiles/``).  Reads settings only.
"""
from __future__ import annotations

import json
import sys


def report() -> dict:
    import torch
    out: dict = {"python": sys.version.split()[0], "torch": torch.__version__,
                 "cuda_build": torch.version.cuda}
    try:
        from .ops._ext import ext
        mod = ext()
        out["extension"] = {"loaded": True, "file": getattr(mod, "__file__", None)}
    except Exception as e:          # reported, not raised: the point is to say what is missing
        mod = None
        out["extension"] = {"loaded": False, "error": f"{type(e).__name__}: {e}"}
    try:
        out["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:
        out["nccl"] = None
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    gpus = []
    for d in range(n):
        p = torch.cuda.get_device_properties(d)
        g = {"index": d, "name": p.name, "capability": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
             "memory_gb": round(p.total_memory / 1e9, 1), "sm_100a": (p.major, p.minor) == (10, 0)}
        if mod is not None:
            try:
                g["multicast"] = bool(mod.multicast_supported(d))
            except Exception as e:
                g["multicast"] = f"unknown ({e})"
        gpus.append(g)
    out["gpus"] = gpus
    if mod is not None and n > 1:
        out["peer_access"] = [[d == e or bool(mod.can_access_peer(d, e)) for e in range(n)] for d in range(n)]
    notes = []
    if not out["extension"]["loaded"]:
        notes.append("build the extension: python setup.py build_ext --inplace")
    if n == 0:
        notes.append("no CUDA device: only cpu_direct can run here")
    elif not all(g["sm_100a"] for g in gpus):
        notes.append("the transfer kernels are built for sm_100a (B200) only")
    if n > 1 and "peer_access" in out and not all(all(r) for r in out["peer_access"]):
        notes.append("some GPU pairs lack peer access: gpu_direct needs it between senders and receivers")
    # the NVLink figures the dry-run planner and the benchmark's roofline divide by
    from .ops.microbench import _mc_peak_gbs, _peer_peak_gbs
    out["measured_link_gbs"] = {"gpu_to_gpu": _peer_peak_gbs(), "multicast_store": _mc_peak_gbs()}
    out["notes"] = notes
    return out


def main() -> int:
    print(json.dumps(report()))
    return 0


if __name__ == "__main__":
    sys.exit(main())
