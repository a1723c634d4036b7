"""weightbridge_b200: trainer -> rollout weight transfer for B200 (sm_100a).

Public API (same names as the reference package ``wbridge``): ``WeightSender``,
``WeightReceiver``, ``WeightReceiverController``, ``WeightData``, ``dtype_str_to_torch``,
``dtype_to_str``.
"""
from .core.shard import WeightData, check_shard_compatibility, shards_iterator, original_total_numel
from .utils.dtypes import dtype_str_to_torch, dtype_to_str

__all__ = [
    "WeightData", "check_shard_compatibility", "shards_iterator", "original_total_numel",
    "dtype_str_to_torch", "dtype_to_str",
]
__version__ = "0.1.0"
