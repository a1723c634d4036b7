"""On-disk cache of planned ops, so a restarted trainer reuses the plans of its last run.

A sender plans one op list per receiver from two address-free descriptions: its own
``relative_binding`` (each bound view is an "allocation" of its own, resolved to the view's
address only when the ops are lowered) and the receiver's physical binding (allocation
indices into the receiver's exported memory, offsets inside them).  The op list is therefore
a pure function of both layouts and of the entry subset, and a file keyed by their hash stays
valid across process restarts and tensor reallocations.  Entries are JSON, written to a
temporary file and renamed into place, so concurrent senders never read a partial file; a
file that does not parse is ignored and rewritten.

The reference has no plan cache: every ``connect`` recomputes and re-sends the overlap
(``wbridge/backend/direct_sender.py:141-158``).
"""
from __future__ import annotations

import hashlib
import json
import os
import tempfile
from typing import Sequence

import torch

from ..utils.dtypes import dtype_str_to_torch, dtype_to_str
from .binding import Binding
from .plan import Op, PhysBinding, PhysShard

FORMAT = 1


def relative_binding(binding: Binding) -> tuple[PhysBinding, list[int]]:
    """The physical binding of ``binding`` with allocation ``i`` standing for the ``i``-th
    bound view (offset 0 inside it), and the views' addresses in that order."""
    pb = PhysBinding(binding.meta)
    ptrs: list[int] = []
    for name, views in binding.entries.items():
        lst = []
        for bs in views:
            lst.append(PhysShard(bs.shard, len(ptrs), 0, list(bs.strides)))
            ptrs.append(bs.tensor.data_ptr())
        pb.entries[name] = lst
    return pb, ptrs


def plan_key(src_json: dict, dst_json: dict, names: Sequence[str] | None) -> str:
    payload = json.dumps([FORMAT, src_json, dst_json, None if names is None else list(names)],
                         sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(payload.encode()).hexdigest()


def _op_to_json(o: Op) -> list:
    return [o.kind, o.name, list(o.src), list(o.dst), list(o.extents), list(o.src_strides), list(o.dst_strides),
            dtype_to_str(o.src_dtype), dtype_to_str(o.dst_dtype), None if o.scale is None else list(o.scale),
            o.scale_strides, None if o.block is None else list(o.block), None if o.key is None else list(o.key)]


def _op_from_json(j: list) -> Op:
    kind, name, src, dst, ext, ss, ds, sd, dd, scale, sstr, block, key = j
    return Op(kind, name, (int(src[0]), int(src[1])), (int(dst[0]), int(dst[1])), [int(x) for x in ext],
              [int(x) for x in ss], [int(x) for x in ds], dtype_str_to_torch(sd), dtype_str_to_torch(dd),
              None if scale is None else (int(scale[0]), int(scale[1])),
              None if sstr is None else [int(x) for x in sstr],
              None if block is None else (int(block[0]), int(block[1])),
              None if key is None else (key[0], int(key[1]), int(key[2])))


class PlanCache:
    """Op lists on disk under ``directory``, one file per plan key."""

    def __init__(self, directory: str):
        self.directory = directory
        self.hits = self.misses = 0

    def _path(self, key: str) -> str:
        return os.path.join(self.directory, f"{key}.json")

    def get(self, key: str) -> list[Op] | None:
        try:
            with open(self._path(key)) as f:
                doc = json.load(f)
            if doc.get("format") != FORMAT or doc.get("key") != key:
                raise ValueError("stale entry")
            ops = [_op_from_json(j) for j in doc["ops"]]
        except (OSError, ValueError, KeyError, TypeError, IndexError):
            self.misses += 1
            return None
        self.hits += 1
        return ops

    def put(self, key: str, ops: Sequence[Op]) -> None:
        os.makedirs(self.directory, exist_ok=True)
        doc = {"format": FORMAT, "key": key, "torch": torch.__version__, "ops": [_op_to_json(o) for o in ops]}
        fd, tmp = tempfile.mkstemp(dir=self.directory, prefix=".plan-", suffix=".tmp")
        try:
            with os.fdopen(fd, "w") as f:
                json.dump(doc, f, separators=(",", ":"))
            os.replace(tmp, self._path(key))
        except BaseException:
            try:
                os.unlink(tmp)
            except OSError:
                pass
            raise
