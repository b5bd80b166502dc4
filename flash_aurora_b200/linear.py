"""Linear layer with a fused bias + exact-GELU epilogue on the tensor cores (``fa_linear_bias_act``).

The block MLP (upstream ``aurora/model/swin3d.py:73-109``) runs fc1 in bf16 and then
``nn.GELU()`` on the (tokens x 4D) hidden tensor. Here both are one kernel: the GELU (the fitted
erfc form of :func:`flash_aurora_b200.gelu_erf`, applied to the fp32 sum before the single bf16
rounding) runs on the epilogue warps while the tensor cores work on the next tile, so the hidden
tensor is written once and never re-read for the activation.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

__all__ = ["linear_bias_act"]

_ACTS = {"gelu": _lib.FA_ACT_GELU, "none": _lib.FA_ACT_NONE}


def linear_bias_act(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, act: str = "gelu",
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``act(x @ weight.T + bias)`` for bf16 CUDA tensors: ``x (..., K)``, ``weight (N, K)``,
    ``bias (N)``; ``N % 256 == 0`` and ``K % 64 == 0``."""
    if act not in _ACTS:
        raise ValueError(f"act must be one of {tuple(_ACTS)}")
    for t, name in ((x, "x"), (weight, "weight"), (bias, "bias")):
        if t.device.type != "cuda" or t.dtype != torch.bfloat16:
            raise ValueError(f"linear_bias_act requires bfloat16 CUDA tensors ({name} is {t.dtype} on {t.device})")
    K = x.shape[-1]
    N = weight.shape[0]
    if weight.shape != (N, K) or bias.shape != (N,):
        raise ValueError(f"weight must be (N, {K}) and bias (N,), got {tuple(weight.shape)} and {tuple(bias.shape)}")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    weight = weight.contiguous()
    bias = bias.contiguous()
    M = x2.shape[0]
    shape = tuple(x.shape[:-1]) + (N,)
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
    elif tuple(out.shape) != shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bfloat16 tensor of shape {shape}")
    rc = _lib.load().fa_linear_bias_act(
        x2.data_ptr(), weight.data_ptr(), bias.data_ptr(), out.data_ptr(), M, N, K, x2.stride(0), K, N,
        _ACTS[act], _lib.stream_ptr(x.device))
    _lib.check(rc, "linear_bias_act")
    return out
