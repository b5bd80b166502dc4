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

__all__ = ["linear_bias_act", "linear_adaln_film_add_residual"]

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


_ROWS = {"tokens": _lib.FA_ROWS_TOKENS, "windows": _lib.FA_ROWS_WINDOWS}


def linear_adaln_film_add_residual(
    a: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    residual: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    res,
    window_size,
    shift_size,
    *,
    rows: str,
    scale_bias: float = 0.0,
    eps: float = 1e-5,
    out_bf16: Optional[torch.Tensor] = None,
    next_windows: Optional[tuple] = None,
) -> torch.Tensor:
    """``residual + LN(bf16(a @ weight.T + bias)) * (scale_bias + scale) + shift`` for D = 512, as one
    kernel (``fa_linear_adaln_film``): the linear's bf16 output never reaches HBM.

    ``rows="windows"``: ``a`` is ``(B * nW, N, K)`` in this block's window layout (the attention
    output before proj); each row lands at its token (crop / un-roll / merge), pad slots are
    dropped; ``out_bf16`` (optional, ``(B, L, 512)`` bf16) receives a bf16 copy.
    ``rows="tokens"``: ``a`` is ``(B, L, K)`` (the MLP hidden before fc2); ``next_windows =
    (next_shift, buffer)`` also writes the result in bf16 into the window layout of a following
    block. ``residual`` is ``(B, L, 512)`` fp32, ``scale``/``shift`` ``(B, 1, 512)`` fp32.
    Returns the fp32 ``(B, L, 512)`` result. Equals ``linear_bias_act`` followed by the matching
    AdaLN op up to the summation order of the fp32 row statistics.
    """
    if rows not in _ROWS:
        raise ValueError(f"rows must be one of {tuple(_ROWS)}")
    for t, name in ((a, "a"), (weight, "weight"), (bias, "bias")):
        if t.device.type != "cuda" or t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be a bfloat16 CUDA tensor")
    B, L, D = residual.shape
    K = a.shape[-1]
    if D != 512 or weight.shape != (512, K) or bias.shape != (512,):
        raise ValueError("linear_adaln_film_add_residual needs 512 output features")
    if residual.dtype != torch.float32 or scale.dtype != torch.float32 or shift.dtype != torch.float32:
        raise ValueError("residual, scale and shift must be float32")
    C, H, W = (int(v) for v in res)
    if L != C * H * W:
        raise ValueError(f"residual has {L} tokens, res {tuple(res)} has {C * H * W}")
    a2 = a.reshape(-1, K)
    if a2.stride(-1) != 1:
        a2 = a2.contiguous()
    weight, bias = weight.contiguous(), bias.contiguous()
    residual = residual.contiguous()
    scale = scale.reshape(B, D).contiguous()
    shift = shift.reshape(B, D).contiguous()
    out = torch.empty_like(residual)
    if out_bf16 is not None and (tuple(out_bf16.shape) != (B, L, D) or out_bf16.dtype != torch.bfloat16
                                 or not out_bf16.is_contiguous()):
        raise ValueError(f"out_bf16 must be a contiguous bfloat16 tensor of shape {(B, L, D)}")
    win = None
    nxt = (0, 0, 0)
    if next_windows is not None:
        nxt, win = next_windows
        if win.dtype != torch.bfloat16 or not win.is_contiguous() or win.shape[-1] != D:
            raise ValueError("the next-block window buffer must be a contiguous bfloat16 (B * nW, N, 512) tensor")
    rc = _lib.load().fa_linear_adaln_film(
        a2.data_ptr(), weight.data_ptr(), bias.data_ptr(), a2.shape[0], K, a2.stride(0), _ROWS[rows],
        scale.data_ptr(), shift.data_ptr(), float(scale_bias), float(eps), residual.data_ptr(), out.data_ptr(),
        out_bf16.data_ptr() if out_bf16 is not None else None, win.data_ptr() if win is not None else None,
        B, C, H, W, _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.i32x3(nxt), _lib.stream_ptr(a.device))
    _lib.check(rc, "linear_adaln_film_add_residual")
    return out
