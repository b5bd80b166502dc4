"""Exact (erf) GELU of the block MLP on the CUDA library (``fa_gelu_erf``).

Upstream applies ``nn.GELU()`` between fc1 and fc2 (``aurora/model/swin3d.py:73-109``). Here it
runs in place on the bf16 fc1 output with 16-byte streaming accesses; the arithmetic is PyTorch's
(``x * 0.5 * (1 + erf(x / sqrt(2)))`` in fp32, rounded to the tensor dtype).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

__all__ = ["gelu_erf"]


def gelu_erf(x: torch.Tensor, out: Optional[torch.Tensor] = None, *, inplace: bool = False) -> torch.Tensor:
    """``GELU(x)`` for a CUDA float32/bfloat16 tensor; ``inplace=True`` overwrites ``x``."""
    if x.device.type != "cuda" or x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("gelu_erf requires a CUDA float32/bfloat16 tensor.")
    if inplace:
        if not x.is_contiguous():
            raise ValueError("in-place gelu_erf needs a contiguous tensor")
        out = x
    else:
        x = x.contiguous()
        if out is None:
            out = torch.empty_like(x)
        elif out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous() or out.device != x.device:
            raise ValueError("out must be a contiguous tensor of x's shape, dtype and device")
    rc = _lib.load().fa_gelu_erf(x.data_ptr(), out.data_ptr(), _lib.dtype_code(x.dtype), x.numel(),
                                 _lib.stream_ptr(x.device))
    _lib.check(rc, "gelu_erf")
    return out
