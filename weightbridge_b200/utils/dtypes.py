"""dtype helpers shared by the metadata, the planner and the kernels.

Parity: ``dtype_str_to_torch`` / ``dtype_to_str`` keep the names and behaviour of
``wbridge/utils/data.py:12-22`` in the reference (short names, ``"torch."`` prefix accepted).
The numeric codes are this library's own wire codes for the device descriptor tables.
"""
from __future__ import annotations

import torch

# Wire codes used in the device descriptor tables (csrc/wb_common.h mirrors them).
DTYPE_CODES: dict[torch.dtype, int] = {
    torch.uint8: 0,
    torch.int8: 1,
    torch.float16: 2,
    torch.bfloat16: 3,
    torch.float32: 4,
    torch.float8_e4m3fn: 5,
    torch.int32: 6,
    torch.int64: 7,
    torch.float64: 8,
    torch.bool: 9,
    torch.int16: 10,
    torch.float8_e5m2: 11,
}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}

# dtypes the cast path converts between (elementwise, round-to-nearest-even).
FLOAT_CAST_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def dtype_str_to_torch(s: str) -> torch.dtype:
    """Map ``"float32"`` / ``"torch.float32"`` to ``torch.float32``."""
    s = s.strip()
    if s.startswith("torch."):
        s = s[len("torch."):]
    dt = getattr(torch, s, None)
    if not isinstance(dt, torch.dtype):
        raise ValueError(f"unknown dtype string {s!r}")
    return dt


def dtype_to_str(dtype: torch.dtype) -> str:
    """Short canonical name of a torch dtype (``torch.bfloat16`` -> ``"bfloat16"``)."""
    return str(dtype).rsplit(".", 1)[-1]


def as_dtype(dtype: torch.dtype | str) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    if isinstance(dtype, str):
        return dtype_str_to_torch(dtype)
    raise TypeError(f"dtype must be a torch.dtype or a string, got {type(dtype).__name__}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"dtype {dtype} has no wire code") from None
