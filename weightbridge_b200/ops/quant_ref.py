"""Plain-PyTorch reference of the conversions the transfer kernels fuse (the oracle).

Block-scaled fp8: a 2-D tensor is cut into ``bn x bk`` blocks (128 x 128 by default; edge
blocks may be partial).  For each block, ``scale = amax / 448`` in fp32 (``scale = 1`` for an
all-zero block), ``inv = 1 / scale`` (IEEE, round to nearest) and
``q = satfinite_e4m3(x * inv)`` with round-to-nearest-even.  The receiver dequantises as
``q * scale``; the scale tensor is what SGLang names ``weight_scale_inv``.  The CUDA kernel
and the C++ CPU executor perform the same IEEE operations, so all three agree bit for bit.
"""
from __future__ import annotations

import torch

FP8_E4M3_MAX = 448.0


def cast_region(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Elementwise cast between float dtypes (round to nearest even)."""
    return x.to(dtype)


def convert_region(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        raise ValueError("fp8 targets need block scales: use block_quant_fp8_ref")
    return cast_region(x, dtype)


def block_scales_shape(n: int, k: int, block: tuple[int, int] = (128, 128)) -> tuple[int, int]:
    bn, bk = block
    return (n + bn - 1) // bn, (k + bk - 1) // bk


def block_quant_fp8_ref(x: torch.Tensor, block: tuple[int, int] = (128, 128)
                        ) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise a 2-D (or batched 3-D) tensor to e4m3 with per-block fp32 scales."""
    if x.dim() == 3:
        qs, ss = zip(*(block_quant_fp8_ref(x[i], block) for i in range(x.shape[0])))
        return torch.stack(qs), torch.stack(ss)
    if x.dim() != 2:
        raise ValueError("block quantisation needs a 2-D tensor")
    bn, bk = block
    n, k = x.shape
    sn, sk = block_scales_shape(n, k, block)
    x32 = x.float()
    pad = torch.zeros(sn * bn, sk * bk, dtype=torch.float32, device=x.device)
    pad[:n, :k] = x32.abs()
    amax = pad.view(sn, bn, sk, bk).amax(dim=(1, 3))
    # tensor / tensor: torch on CUDA turns a division by a Python scalar into a multiply by
    # the reciprocal, which rounds differently from the IEEE division the kernel performs
    scale = torch.where(amax > 0, amax / torch.full_like(amax, FP8_E4M3_MAX), torch.ones_like(amax))
    inv = torch.ones_like(scale) / scale
    full = inv.repeat_interleave(bn, 0).repeat_interleave(bk, 1)[:n, :k]
    q = (x32 * full).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q, scale


def block_dequant_fp8_ref(q: torch.Tensor, scale: torch.Tensor,
                          block: tuple[int, int] = (128, 128)) -> torch.Tensor:
    if q.dim() == 3:
        return torch.stack([block_dequant_fp8_ref(q[i], scale[i], block) for i in range(q.shape[0])])
    bn, bk = block
    n, k = q.shape
    full = scale.repeat_interleave(bn, 0).repeat_interleave(bk, 1)[:n, :k]
    return q.float() * full
