"""Model architecture descriptors and deterministic synthetic weights."""
from .arch import PRESETS, ModelArch, get_arch

__all__ = ["PRESETS", "ModelArch", "get_arch"]
