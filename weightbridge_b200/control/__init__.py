"""Control plane: sender, receiver worker, HTTP controller, session store, assignment."""
from .controller import WeightReceiverController
from .receiver import WeightReceiver
from .sender import SyncStats, WeightSender

__all__ = ["WeightReceiverController", "WeightReceiver", "SyncStats", "WeightSender"]
