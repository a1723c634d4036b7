"""Loader of the in-tree native extension ``weightbridge_b200._C``.

The extension holds the sm_100a transfer kernel, the CPU executor and the IPC/VMM/multicast
wrappers.  There is no fallback: if it is missing, every native op raises with the build
command, so a GPU run can never silently take a slower path.
"""
from __future__ import annotations

_C = None
_ERR: Exception | None = None


def ext():
    global _C, _ERR
    if _C is None and _ERR is None:
        try:
            from .. import _C as mod  # type: ignore[attr-defined]
            _C = mod
        except ImportError as e:  # pragma: no cover - exercised only when unbuilt
            _ERR = e
    if _C is None:
        raise RuntimeError(
            "weightbridge_b200 native extension is not built "
            f"({_ERR}); run `python setup.py build_ext --inplace` in the repository root")
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
