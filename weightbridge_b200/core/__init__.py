"""Shard algebra, bindings and the transfer planner."""
from .shard import (WeightData, TensorBridge, align_shards, box_copies, box_copy, check_shard_compatibility,
                    _check_shard_compatibility, coalesce, normalize_shards, original_total_numel,
                    refine, shard_extents, shard_numel, shards_iterator)
from .binding import Binding, BoundShard, bind, pack_into, unpack_from

__all__ = ["WeightData", "TensorBridge", "align_shards", "box_copies", "box_copy", "check_shard_compatibility",
           "_check_shard_compatibility", "coalesce", "normalize_shards", "original_total_numel", "refine",
           "shard_extents", "shard_numel", "shards_iterator", "Binding", "BoundShard", "bind", "pack_into",
           "unpack_from"]
