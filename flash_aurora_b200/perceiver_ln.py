"""Perceiver decoder LayerNorm (+ residual) on the C ABI.

Drop-in for upstream ``aurora/ops/triton_perceiver_ln.py``: ``layernorm_affine_forward``
(:25-32) and ``layernorm_affine_add_residual_forward`` (:35-47), which
``aurora/model/perceiver.py:255-276`` calls for the post-norm ``ln1(attn(...)) + latents`` and
``ln2(ff(...)) + latents`` of each ``PerceiverResampler`` layer. Same arguments, output dtype and
exceptions; the kernel is ``fa_layernorm_affine`` (``csrc/layernorm.cu``).

Numerics: ``LayerNorm(x) * weight + bias (+ residual)`` in fp32 with one rounding to ``x``'s dtype,
like upstream's fused kernel. The variance is taken about the mean from registers (the
``nn.LayerNorm`` form) rather than upstream's ``E[x^2] - mean^2``. A residual of another dtype than
``x`` is converted to ``x``'s dtype first (upstream adds it in fp32 as loaded).
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["layernorm_affine_forward", "layernorm_affine_add_residual_forward"]

_MAX_D = 4096


def layernorm_affine_forward(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """``nn.LayerNorm(D)`` with affine weight and bias on the last dimension of ``(B, L, D)``."""
    return _dispatch(x, None, weight, bias, float(eps))


def layernorm_affine_add_residual_forward(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                                          bias: torch.Tensor, eps: float) -> torch.Tensor:
    """``layer_norm(x) * weight + bias + residual``; ``x`` and ``residual`` are ``(B, L, D)``."""
    if residual.shape != x.shape:
        raise ValueError("residual must match x shape.")
    return _dispatch(x, residual, weight, bias, float(eps))


def _code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return _lib.FA_F32
    if dt == torch.bfloat16:
        return _lib.FA_BF16
    if dt == torch.float16:
        return _lib.FA_F16
    raise ValueError(f"Unsupported dtype {dt}; use float16, bfloat16, or float32.")


def _dispatch(x: torch.Tensor, residual, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    if x.device.type != "cuda":
        raise ValueError("perceiver LayerNorm ops require CUDA tensors.")
    if x.dim() != 3:
        raise ValueError(f"Expected x (B, L, D), got shape {tuple(x.shape)}.")
    B, L, D = x.shape
    if D > _MAX_D:
        raise ValueError(f"D must be <= {_MAX_D}, got {D}.")
    if weight.shape != (D,) or bias.shape != (D,):
        raise ValueError("weight and bias must be shape (D,).")
    code = _code(x.dtype)
    for t, name in ((weight, "weight"), (bias, "bias")):
        if t.device != x.device:
            raise ValueError(f"{name} must be on {x.device}")
    if weight.dtype != bias.dtype:  # widen both (exact for bf16 / fp16)
        weight, bias = weight.float(), bias.float()
    wcode = _code(weight.dtype)
    x = x.contiguous()
    weight, bias = weight.contiguous(), bias.contiguous()
    if residual is not None:
        if residual.device != x.device:
            raise ValueError(f"residual must be on {x.device}")
        residual = residual.to(x.dtype).contiguous()
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    rows = B * L
    if rows == 0:
        return out
    lib = _lib.load()
    _lib.check(lib.fa_layernorm_affine(x.data_ptr(), code, residual.data_ptr() if residual is not None else None,
                                       weight.data_ptr(), bias.data_ptr(), wcode, eps, out.data_ptr(), rows, D,
                                       _lib.stream_ptr(x.device)), "fa_layernorm_affine")
    return out
