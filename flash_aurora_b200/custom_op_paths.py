"""Gating predicates of the fused Swin3D operators, under the upstream names.

Upstream (``flash_aurora/aurora/model/custom_op_paths.py:501-579``) asks these predicates before
each fused call and falls back to eager PyTorch when one says no. This package has no fallback,
so here each predicate answers a narrower question: does the B200 operator of this package accept
this input? It keeps upstream's conditions (enabled, inference mode, no dropout, CUDA, dtype,
packed-QKV layout) and adds the ones the B200 kernels impose: the in-tree CUDA library is built, the
tensor sits on an sm_100 device, and for attention the window holds at most 144 tokens with
head_dim 64. A caller that gets ``False`` must not call the operator (it would raise).
"""

from __future__ import annotations

import os

import torch

from . import _lib

__all__ = [
    "b200_available",
    "can_use_triton_layout",
    "can_use_triton_adaln",
    "can_use_triton_gelu",
    "can_use_cute_window_attention",
    "can_use_cute_qkvpacked",
]

_ELEM_DTYPES = (torch.float32, torch.bfloat16)
_MAX_TOKENS = 144
_HEAD_DIM = 64


def b200_available(t: torch.Tensor) -> bool:
    """``t`` is a CUDA tensor on an sm_100 (B200-class) device and the CUDA library is built."""
    if not t.is_cuda or not os.path.exists(_lib.LIB_PATH):
        return False
    return torch.cuda.get_device_capability(t.device)[0] == 10


def can_use_triton_layout(x: torch.Tensor, *, enabled: bool) -> bool:
    """Roll/pad/partition and its inverse (``swin3d_layout``): fp32 or bf16 on the device."""
    return bool(enabled) and x.dtype in _ELEM_DTYPES and b200_available(x)


def can_use_triton_adaln(x: torch.Tensor, *, enabled: bool, training: bool, drop_path_is_identity: bool) -> bool:
    """Fused AdaLN + FiLM (+ residual) on fp32 activations, inference only."""
    return (bool(enabled) and not training and drop_path_is_identity and x.dtype == torch.float32
            and b200_available(x))


def can_use_triton_gelu(x: torch.Tensor, *, enabled: bool, training: bool, drop_p: float) -> bool:
    """Exact GELU (``gelu_erf``) on fp32 or bf16, inference only, no dropout."""
    return (bool(enabled) and not training and drop_p == 0.0 and x.dtype in _ELEM_DTYPES
            and b200_available(x))


def _window_tokens(qkv: torch.Tensor) -> int | None:
    """Tokens per window of a packed ``(Bwin, N, 3C)`` or split ``(Bwin, H, N, Dh)`` tensor."""
    if qkv.ndim == 3:
        return int(qkv.shape[1])
    if qkv.ndim == 4:
        return int(qkv.shape[2])
    return None


def can_use_cute_window_attention(qkv: torch.Tensor, *, enabled: bool, training: bool,
                                  attn_dropout: float) -> bool:
    """Window attention: fp32 or bf16, no grad, no dropout, at most 144 tokens per window."""
    n = _window_tokens(qkv)
    return (bool(enabled) and not training and attn_dropout == 0.0 and qkv.dtype in _ELEM_DTYPES
            and not torch.is_grad_enabled() and n is not None and 1 <= n <= _MAX_TOKENS
            and b200_available(qkv))


def can_use_cute_qkvpacked(qkv: torch.Tensor, *, num_heads: int, head_dim: int, cute_enabled: bool,
                           training: bool, attn_dropout: float) -> bool:
    """Packed-QKV attention: the contiguous ``Linear(D, 3D)`` output ``(Bwin, N, 3 * H * 64)``."""
    return (can_use_cute_window_attention(qkv, enabled=cute_enabled, training=training, attn_dropout=attn_dropout)
            and qkv.is_contiguous() and qkv.ndim == 3 and head_dim == _HEAD_DIM
            and qkv.shape[-1] == 3 * num_heads * head_dim)
