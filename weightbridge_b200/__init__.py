"""weightbridge_b200: trainer -> rollout weight transfer for B200 (sm_100a).

Public API (the names of the reference package ``wbridge``, ``wbridge/__init__.py:3-17``):
``WeightSender``, ``WeightReceiver``, ``WeightReceiverController``, ``WeightData``,
``dtype_str_to_torch``, ``dtype_to_str``; plus ``TransferConfig`` and the layout adapters
``MegatronLayout`` / ``FSDPLayout`` (trainers) and ``SGLangLayout`` (rollout).
"""
from .core.shard import (WeightData, check_shard_compatibility, original_total_numel,
                         shards_iterator)
from .utils.config import TransferConfig
from .utils.dtypes import dtype_str_to_torch, dtype_to_str


def __getattr__(name):
    # the control plane pulls in zmq/fastapi; import it on first use
    if name in ("WeightSender", "WeightReceiver", "WeightReceiverController", "SyncStats"):
        from . import control
        return getattr(control, name)
    if name == "MegatronLayout":
        from .parallel.megatron import MegatronLayout
        return MegatronLayout
    if name in ("FSDPLayout", "HFLayout"):
        from .parallel import fsdp
        return getattr(fsdp, name)
    if name in ("SGLangLayout", "VLLMLayout"):
        from .parallel import sglang
        return getattr(sglang, name)
    raise AttributeError(name)


__all__ = [
    "WeightData", "WeightSender", "WeightReceiver", "WeightReceiverController", "TransferConfig",
    "check_shard_compatibility", "shards_iterator", "original_total_numel", "dtype_str_to_torch",
    "dtype_to_str", "MegatronLayout", "FSDPLayout", "HFLayout", "SGLangLayout", "VLLMLayout",
]
__version__ = "0.1.0"
