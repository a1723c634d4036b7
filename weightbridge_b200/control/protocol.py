"""Control-plane messages and state shared by sender, controller and receiver workers.

Parity: the message names, the ``ConnectRequest`` fields and the receiver state machine
follow ``wbridge/frontend/receiver.py:23-45``.  Added: a session id (so a stale worker
cannot join a newer session) and the transfer mode in place of the raw backend name.
"""
from __future__ import annotations

import base64
import json
from enum import Enum
from typing import Any, Optional

from pydantic import BaseModel

METADATA_REQUEST = "metadata_request"
CONNECT_REQUEST = "connect_request"
RECEIVE_REQUEST = "receive_request"
STATS_REQUEST = "stats_request"
UPDATE_REQUEST = "update_request"
STOP_REQUEST = "stop_request"

# Version of the sender <-> receiver session protocol (session keys, arm channel, split-block
# amax exchange, the same-host handshake board, the pull direction's rules).  A receiver refuses
# a connect from a sender speaking another version.
PROTOCOL_VERSION = 4


class ReceiverState(str, Enum):
    DISCONNECTED = "disconnected"
    CONNECTING = "connecting"
    CONNECTED = "connected"
    AWAITING_SCHEDULER_UPDATE = "awaiting_scheduler_update"
    FAILED = "failed"


class ConnectRequest(BaseModel):
    master_address: str
    master_port: int
    base_rank: int
    world_size: int
    group_name: str
    sender_world_size: int
    backend: str = "gpu_direct"          # transfer mode: gpu_direct | nvls | nccl | cpu_direct ("gloo" = cpu_direct)
    session: Optional[str] = None
    protocol: int = 1                    # PROTOCOL_VERSION of the sender (absent: an older sender)


def gpu_id(device) -> str | None:
    """A process-independent name of the GPU behind ``device`` (its UUID, base64; the index
    depends on CUDA_VISIBLE_DEVICES), or None for host memory or when it cannot be read."""
    import torch
    dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
    if dev.type != "cuda":
        return None
    try:
        from ..ops._ext import ext
        return b64(ext().device_uuid(dev.index if dev.index is not None else torch.cuda.current_device()))
    except Exception:
        return None


def b64(data: bytes) -> str:
    return base64.b64encode(data).decode("ascii")


def unb64(s: str) -> bytes:
    return base64.b64decode(s.encode("ascii"))


def dumps(obj: Any) -> bytes:
    return json.dumps(obj, separators=(",", ":")).encode("utf-8")


def loads(data: bytes | str) -> Any:
    return json.loads(data)
