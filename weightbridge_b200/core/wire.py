"""Wire chunks: the packed overlap of one (sender, receiver) pair cut into bounded messages.

The wire modes (``cpu_direct`` over gloo, ``nccl``) move each pair's overlap as packed
buffers.  Cutting it into chunks of whole entries bounds the buffer memory on both sides to
two chunks per peer (double buffering: one chunk is packed while the previous one is on the
wire) instead of the whole overlap, which for a 70B model at TP 8 is 17.6 GB per pair on each
side.  Both sides cut the same overlap ``WeightData`` with the same rule, so they agree on
every chunk's entries, layout and size without exchanging anything.  The reference sends one
buffer of the whole overlap per pair (``wbridge/utils/data.py:295-320``).
"""
from __future__ import annotations

from .shard import WeightData


def wire_chunks(overlap: WeightData, chunk_bytes: int) -> list[WeightData]:
    """Consecutive groups of ``overlap``'s entries of at most ``chunk_bytes`` each (an entry
    larger than that is a chunk of its own; ``chunk_bytes <= 0``: one chunk).  A quantised
    entry and its scale entry always share a chunk: the pack writes both."""
    units: list[list[str]] = []
    scale_of = {}
    for name in overlap.names():
        q = overlap.quant(name)
        if q and q.get("role") != "scale" and q.get("scale") in overlap:
            scale_of[name] = q["scale"]
    owned = set(scale_of.values())
    for name in overlap.names():
        if name in owned:
            continue
        units.append([name] + ([scale_of[name]] if name in scale_of else []))
    sizes = {n: nbytes for n, nbytes in _entry_bytes(overlap)}
    chunks: list[list[str]] = []
    cur: list[str] = []
    cur_bytes = 0
    for unit in units:
        b = sum(sizes[n] for n in unit)
        if cur and chunk_bytes > 0 and cur_bytes + b > chunk_bytes:
            chunks.append(cur)
            cur, cur_bytes = [], 0
        cur += unit
        cur_bytes += b
    if cur:
        chunks.append(cur)
    js = overlap.to_jsonable()
    return [WeightData({n: js[n] for n in names}) for names in chunks]


def _entry_bytes(overlap: WeightData):
    for start, end, name, _shards, _dtype in overlap.iter_with_intv():
        yield name, end - start


def restrict_overlap(overlap: WeightData, names) -> WeightData:
    """``overlap`` limited to the entries ``names`` (a partial sync), with the scale entries of
    the quantised ones."""
    keep = set(names)
    js = overlap.to_jsonable()
    out = {}
    for n, e in js.items():
        q = e.get("quant") or {}
        if n in keep or (q.get("role") == "scale" and q.get("of") in keep):
            out[n] = e
    return WeightData(out)


def buffer_bytes(overlap: WeightData, chunk_bytes: int) -> int:
    """Size of a wire buffer that holds any chunk of ``overlap`` or of any subset of its
    entries: a chunk is at most ``chunk_bytes`` or one unit (an entry with its scales), and
    never more than the whole overlap."""
    total = overlap.total_nbytes()
    if chunk_bytes <= 0:
        return max(1, total)
    sizes = {n: b for n, b in _entry_bytes(overlap)}
    unit = 0
    for name in overlap.names():
        q = overlap.quant(name) or {}
        if q.get("role") == "scale":
            continue
        unit = max(unit, sizes[name] + (sizes.get(q["scale"], 0) if q.get("scale") else 0))
    return max(1, min(total, max(chunk_bytes, unit)))
