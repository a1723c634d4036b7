"""Deterministic synthetic weights: N(0, std) values addressed by logical element index.

Every element of a logical HF tensor gets a value that depends only on (seed, tensor name,
flat logical index), so each rank can fill its own shard (any box, any factorisation, any
strided view) without materialising the full tensor, and a receiver can regenerate what it
should have received and compare bit for bit.  Uses a 32-bit integer mixing hash and a
Box-Muller transform.  On a CUDA device one launch of the native fill kernel
(``csrc/wb_synth.cu``) writes a whole view; ``synth_values`` states the same arithmetic in
torch ops, which the host path runs and the GPU tests compare the kernel against bit for bit.
"""
from __future__ import annotations

import math
import zlib
from typing import Sequence

import torch

from ..core.shard import Shard

_M = 0x45D9F3B
_MASK = 0xFFFFFFFF


def _mix32(x: torch.Tensor) -> torch.Tensor:
    x = (((x >> 16) ^ x) * _M) & _MASK
    x = (((x >> 16) ^ x) * _M) & _MASK
    return (x >> 16) ^ x


def name_key(name: str, seed: int = 0) -> int:
    return (zlib.crc32(name.encode()) ^ ((seed * 0x9E3779B1) & _MASK)) & _MASK


def logical_index(box: Shard, device, start: int = 0, stop: int | None = None) -> torch.Tensor:
    """Flat row-major logical index of every element of ``box`` rows [start, stop) of dim 0."""
    widths = [w for _, _, w in box]
    lstr = [1] * len(box)
    for d in range(len(box) - 2, -1, -1):
        lstr[d] = lstr[d + 1] * widths[d + 1]
    idx = None
    for d, (l, r, _w) in enumerate(box):
        lo, hi = (l + start, l + (stop if stop is not None else r - l)) if d == 0 else (l, r)
        a = torch.arange(lo, hi, device=device, dtype=torch.int64) * lstr[d]
        shape = [1] * len(box)
        shape[d] = hi - lo
        a = a.view(shape)
        idx = a if idx is None else idx + a
    return idx


def synth_values(name: str, box: Shard, device, dtype=torch.float32, seed: int = 0, std: float = 0.02,
                 start: int = 0, stop: int | None = None) -> torch.Tensor:
    idx = logical_index(box, device, start, stop)
    key = name_key(name, seed)
    hi = _mix32((idx >> 32) ^ key)
    h1 = _mix32((idx & _MASK) ^ hi)
    h2 = _mix32(h1 ^ 0x68E31DA4)
    u1 = (h1.to(torch.float64) + 1.0) / 4294967297.0
    u2 = h2.to(torch.float64) / 4294967296.0
    z = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)
    return (z * std).to(dtype)


def _native_fill(view: torch.Tensor, name: str, box: Shard, seed: int, std: float) -> bool:
    """One launch of the fill kernel on the view's device and current stream; False when the
    view's dtype is not one the kernel writes."""
    from ..ops._ext import ext
    from ..utils.dtypes import DTYPE_CODES
    code = DTYPE_CODES.get(view.dtype)
    if code is None or not ext().synth_dtype_supported(code) or len(box) > 8:
        return False
    widths = [w for _, _, w in box]
    lstr = [1] * len(box)
    for d in range(len(box) - 2, -1, -1):
        lstr[d] = lstr[d + 1] * widths[d + 1]
    stream = torch.cuda.current_stream(view.device).cuda_stream
    with torch.cuda.device(view.device):
        ext().synth_fill(view.data_ptr(), code, name_key(name, seed), float(std), list(view.shape),
                         list(view.stride()), [l for l, _, _ in box], lstr, stream)
    return True


def synth_fill(view: torch.Tensor, name: str, box: Shard, seed: int = 0, std: float = 0.02,
               chunk_elems: int = 1 << 25) -> torch.Tensor:
    """Fill ``view`` (shape == box extents, any strides) with the synthetic values."""
    ext = [r - l for l, r, _ in box]
    if list(view.shape) != ext:
        view = view.view(ext)
    if view.is_cuda and view.numel() and _native_fill(view, name, box, seed, std):
        return view
    rows = ext[0]
    per_row = max(1, view.numel() // max(rows, 1))
    step = max(1, chunk_elems // per_row)
    for s in range(0, rows, step):
        e = min(rows, s + step)
        view[s:e].copy_(synth_values(name, box, view.device, view.dtype, seed, std, s, e))
    return view


def synth_full(name: str, shape: Sequence[int], dtype=torch.float32, device="cpu", seed: int = 0,
               std: float = 0.02) -> torch.Tensor:
    box = [(0, int(d), int(d)) for d in shape]
    t = torch.empty(list(shape), dtype=dtype, device=device)
    return synth_fill(t, name, box, seed, std)
