"""Parallel layouts (Megatron trainer, SGLang rollout) and cross-process GPU memory."""
