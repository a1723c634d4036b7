"""The reference's ``wbridge.frontend`` names: ``WeightSender``, ``WeightReceiver``,
``WeightReceiverController`` (``wbridge/frontend/__init__.py:3-6``)."""
from .control import WeightReceiver, WeightReceiverController, WeightSender

__all__ = ["WeightReceiver", "WeightReceiverController", "WeightSender"]
