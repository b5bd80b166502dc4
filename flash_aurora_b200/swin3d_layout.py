"""Fused Swin3D window layout: cyclic shift + zero pad + 3D window partition, and its inverse.

Drop-in for upstream ``flash_aurora/aurora/ops/triton_swin3d_layout.py`` (same names through
the ``*_triton`` aliases, same argument meaning, same ``ValueError`` on non-CUDA or
non-float32/bfloat16 input). The work is done by ``fa_roll_pad_partition`` /
``fa_crop_roll_unmerge`` of the CUDA library; ``out_dtype`` additionally lets the partition
write bfloat16 windows straight from a float32 residual stream (round to nearest even, the same
value the upstream bf16 autocast produces when it casts the windows before the QKV linear).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .util import window_geometry
from .workspace_pool import InferenceWorkspacePool

__all__ = [
    "roll_pad_partition_windows",
    "crop_roll_unmerge_windows",
    "roll_pad_partition_windows_triton",
    "crop_roll_unmerge_windows_triton",
]

_DTYPES = (torch.float32, torch.bfloat16)


def roll_pad_partition_windows(
    x: torch.Tensor,
    res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    pool: Optional[InferenceWorkspacePool] = None,
    *,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """``x (B, C, H, W, D)`` -> windows ``(B * nW, N, D)`` (upstream triton_swin3d_layout.py:58-121)."""
    if x.device.type != "cuda" or x.dtype not in _DTYPES:
        raise ValueError("roll_pad_partition_windows requires CUDA float32/bfloat16 input.")
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if out_dtype not in _DTYPES:
        raise ValueError("out_dtype must be float32 or bfloat16")
    B, C, H, W, D = x.shape
    if (C, H, W) != tuple(res):
        raise ValueError(f"x spatial shape {(C, H, W)} does not match res {tuple(res)}")
    x = x.contiguous()
    _, _, _, _, nW, N = window_geometry(tuple(res), tuple(window_size), tuple(shift_size))
    shape = (B * nW, N, D)
    if pool is not None:
        out = pool.get("partition", shape, device=x.device, dtype=out_dtype)
    else:
        out = torch.empty(shape, device=x.device, dtype=out_dtype)
    rc = _lib.load().fa_roll_pad_partition(
        x.data_ptr(), _lib.dtype_code(x.dtype), out.data_ptr(), _lib.dtype_code(out_dtype),
        B, C, H, W, D, _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.stream_ptr(x.device))
    _lib.check(rc, "roll_pad_partition_windows")
    return out


def crop_roll_unmerge_windows(
    windows: torch.Tensor,
    res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    pool: Optional[InferenceWorkspacePool] = None,
    *,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Windows ``(B * nW, N, D)`` -> ``(B, C, H, W, D)`` (upstream triton_swin3d_layout.py:124-189)."""
    if windows.device.type != "cuda" or windows.dtype not in _DTYPES:
        raise ValueError("crop_roll_unmerge_windows requires CUDA float32/bfloat16 input.")
    out_dtype = windows.dtype if out_dtype is None else out_dtype
    if out_dtype not in _DTYPES:
        raise ValueError("out_dtype must be float32 or bfloat16")
    BnW, N, D = windows.shape
    C, H, W = res
    _, _, _, _, nW, Nw = window_geometry(tuple(res), tuple(window_size), tuple(shift_size))
    if BnW % nW != 0:
        raise ValueError(f"window batch {BnW} is not a multiple of the {nW} windows of res {tuple(res)}")
    if N != Nw:
        raise ValueError(f"windows hold {N} tokens, geometry expects {Nw}")
    B = BnW // nW
    windows = windows.contiguous()
    shape = (B, C, H, W, D)
    if pool is not None:
        out = pool.get("unmerge", shape, device=windows.device, dtype=out_dtype)
    else:
        out = torch.empty(shape, device=windows.device, dtype=out_dtype)
    rc = _lib.load().fa_crop_roll_unmerge(
        windows.data_ptr(), _lib.dtype_code(windows.dtype), out.data_ptr(), _lib.dtype_code(out_dtype),
        B, C, H, W, D, _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.stream_ptr(windows.device))
    _lib.check(rc, "crop_roll_unmerge_windows")
    return out


# Upstream names (drop-in for the ``use_triton_layout`` call sites, swin3d.py:742-756).
roll_pad_partition_windows_triton = roll_pad_partition_windows
crop_roll_unmerge_windows_triton = crop_roll_unmerge_windows
