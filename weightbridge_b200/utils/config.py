"""Transfer configuration (dataclass + ``WBRIDGE_*`` environment overrides).

The reference has no configuration beyond constructor arguments (``transfer_mode`` in
``wbridge/frontend/sender.py:15-20``, ``ConnectRequest`` in ``wbridge/frontend/receiver.py:38-45``)
and derives ports from ``CUDA_VISIBLE_DEVICES`` (``wbridge/utils/distributed.py:24-25``).
Here every wait has a deadline and the rendezvous port is chosen by the OS unless given.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, fields

MODE_ALIASES = {
    "gpu_direct": "gpu_direct", "p2p": "gpu_direct", "ipc": "gpu_direct", "ipc_local": "gpu_direct",
    "cpu_direct": "cpu_direct", "cpu": "cpu_direct", "gloo": "cpu_direct",
    "nvls": "nvls", "multicast": "nvls",
    "nccl": "nccl", "nccl_wire": "nccl",
    "auto": "auto",          # chosen at connect: gpu_direct, nccl or cpu_direct (see WeightSender)
}

# modes whose payload travels as packed wire buffers over a process group
WIRE_MODES = ("cpu_direct", "nccl")


def normalize_mode(mode: str) -> str:
    try:
        return MODE_ALIASES[mode]
    except KeyError:
        raise ValueError(f"Invalid transfer mode: {mode!r} (expected one of {sorted(MODE_ALIASES)})") from None


@dataclass
class TransferConfig:
    mode: str = "gpu_direct"
    master_address: str = "auto"          # session store address (sender rank 0); auto: loopback when
                                          # every receiver URL is local, else this host's address
    master_port: int = 0                  # 0: let the OS pick a free port
    connect_timeout_s: float = 120.0      # rendezvous, metadata exchange, plan agreement
    sync_timeout_s: float = 300.0         # one send()/request_update() round
    http_timeout_s: float = 60.0
    zmq_timeout_s: float = 60.0
    kernel_mode: int = -1                 # -1 auto, 0 vector, 1/2/3 TMA bulk pipeline depths
    piece_bytes: int = 16384
    item_bytes: int = 1 << 19
    wire_chunk_bytes: int = 256 << 20     # wire modes: message size per peer (two buffers of it per peer); 0: whole overlap
    grid: int = 0                         # 0: sized from the SM count
    verify_flags: bool = True             # receiver checks every sender's epoch flag
    load_balance: bool = True             # spread replicated shards over senders
    validate_plan: bool = True            # check every work row against registered memory before upload
    require_full_coverage: bool = False   # connect fails (instead of warning) if a rollout entry has no sender
    direction: str = "pull"               # gpu_direct: pull (receivers load the copies; fp8 blocks are still
                                          # quantised and pushed by the senders) | push (senders store all)
    link_gbs: float = 788.0               # per-GPU link bandwidth for the stats' fraction (measured peer peak)
    arm: str = "direct"                   # how each sync is armed: direct (one ZMQ message from sender rank 0
                                          # to every receiver worker) | http (POST /wbridge/receive per sync)
    plan_cache_dir: str = ""              # senders keep their planned ops here across restarts ("": memory only)

    def __post_init__(self):
        self.mode = normalize_mode(self.mode)
        if self.direction not in ("push", "pull"):
            raise ValueError(f"direction must be 'push' or 'pull', not {self.direction!r}")
        if self.arm not in ("direct", "http"):
            raise ValueError(f"arm must be 'direct' or 'http', not {self.arm!r}")

    @staticmethod
    def from_env(**overrides) -> "TransferConfig":
        kw = {}
        for f in fields(TransferConfig):
            v = os.environ.get("WBRIDGE_" + f.name.upper())
            if v is None:
                continue
            if f.type in ("int", int):
                kw[f.name] = int(v)
            elif f.type in ("float", float):
                kw[f.name] = float(v)
            elif f.type in ("bool", bool):
                kw[f.name] = v.lower() in ("1", "true", "yes", "on")
            else:
                kw[f.name] = v
        kw.update({k: v for k, v in overrides.items() if v is not None})
        return TransferConfig(**kw)
