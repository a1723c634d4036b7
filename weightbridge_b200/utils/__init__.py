"""Small shared helpers: dtypes, timing, config, NVTX."""
from .dtypes import dtype_str_to_torch, dtype_to_str

__all__ = ["dtype_str_to_torch", "dtype_to_str"]
