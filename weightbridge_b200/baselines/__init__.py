"""Baselines the transfer kernels are compared against (not used by the library itself)."""
