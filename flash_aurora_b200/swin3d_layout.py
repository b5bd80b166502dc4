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
from .util import band_geometry, window_geometry
from .workspace_pool import InferenceWorkspacePool

__all__ = [
    "roll_pad_partition_windows",
    "crop_roll_unmerge_windows",
    "roll_pad_partition_windows_triton",
    "crop_roll_unmerge_windows_triton",
    "roll_pad_partition_windows_band",
    "band_halo_extract",
    "crop_roll_unmerge_windows_band",
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


# ---------------------------------------------------------------------------------------------
# Latitude bands (a field sharded along H across ranks; see ``flash_aurora_b200.sharding``).
# ---------------------------------------------------------------------------------------------


def _check_halo(halo, B, C, s, W, D, dtype, device, name):
    if s == 0:
        return None
    if halo is None:
        raise ValueError(f"a band with an H shift of {s} rows needs {name}")
    if tuple(halo.shape) != (B, C, s, W, D) or halo.dtype != dtype or halo.device != device:
        raise ValueError(f"{name} must be a {dtype} tensor of shape {(B, C, s, W, D)} on {device}, "
                         f"got {halo.dtype} {tuple(halo.shape)} on {halo.device}")
    return halo.contiguous()


def roll_pad_partition_windows_band(
    x: torch.Tensor,
    halo: Optional[torch.Tensor],
    field_res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    *,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Windows of one latitude band: ``x (B, C, H_band, W, D)`` + ``halo (B, C, s, W, D)`` (the next
    band's first ``s = shift_h`` rows) -> ``(B * nW_band, N, D)``, equal to rows
    ``[h1_begin, h1_end)`` of the field's ``roll_pad_partition_windows``. The halo may be in
    ``x``'s dtype or already in ``out_dtype`` (the neighbour rounded it before sending; the result
    is the same bit for bit; for fp32 ``x`` and bf16 windows)."""
    if x.device.type != "cuda" or x.dtype not in _DTYPES:
        raise ValueError("roll_pad_partition_windows_band requires CUDA float32/bfloat16 input.")
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if out_dtype not in _DTYPES:
        raise ValueError("out_dtype must be float32 or bfloat16")
    B, C, Hb, W, D = x.shape
    ws, ss, nW, N = band_geometry((C, Hb, W), field_res, window_size, shift_size)
    pre_rounded = (halo is not None and halo.dtype == out_dtype == torch.bfloat16 and x.dtype == torch.float32)
    halo_dtype = out_dtype if pre_rounded else x.dtype
    halo = _check_halo(halo, B, C, ss[1], W, D, halo_dtype, x.device, "halo")
    x = x.contiguous()
    out = torch.empty((B * nW, N, D), device=x.device, dtype=out_dtype)
    rc = _lib.load().fa_roll_pad_partition_band(
        x.data_ptr(), halo.data_ptr() if halo is not None else None, _lib.dtype_code(x.dtype),
        _lib.dtype_code(halo_dtype), out.data_ptr(), _lib.dtype_code(out_dtype), B, C, Hb, field_res[1], W, D,
        _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.stream_ptr(x.device))
    _lib.check(rc, "roll_pad_partition_windows_band")
    return out


def band_halo_extract(
    windows: torch.Tensor,
    band_res: tuple[int, int, int],
    field_res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    *,
    out_dtype: Optional[torch.dtype] = None,
    out: Optional[torch.Tensor] = None,
) -> Optional[torch.Tensor]:
    """The band's last ``s`` shifted rows, un-rolled in C and W: ``(B, C, s, W, D)``. They are the
    next band's first ``s`` original rows. ``None`` when the block has no H shift."""
    if windows.device.type != "cuda" or windows.dtype not in _DTYPES:
        raise ValueError("band_halo_extract requires CUDA float32/bfloat16 windows.")
    out_dtype = windows.dtype if out_dtype is None else out_dtype
    C, Hb, W = (int(v) for v in band_res)
    ws, ss, nW, N = band_geometry(band_res, field_res, window_size, shift_size)
    if ss[1] == 0:
        return None
    BnW, Nw, D = windows.shape
    if BnW % nW or Nw != N:
        raise ValueError(f"windows {tuple(windows.shape)} do not match the band's {nW} windows of {N} tokens")
    B = BnW // nW
    shape = (B, C, ss[1], W, D)
    if out is None:
        out = torch.empty(shape, device=windows.device, dtype=out_dtype)
    elif tuple(out.shape) != shape or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {out_dtype} tensor of shape {shape}")
    windows = windows.contiguous()
    rc = _lib.load().fa_band_halo_extract(
        windows.data_ptr(), _lib.dtype_code(windows.dtype), out.data_ptr(), _lib.dtype_code(out_dtype),
        B, C, Hb, field_res[1], W, D, _lib.i32x3(window_size), _lib.i32x3(shift_size),
        _lib.stream_ptr(windows.device))
    _lib.check(rc, "band_halo_extract")
    return out


def crop_roll_unmerge_windows_band(
    windows: torch.Tensor,
    halo_in: Optional[torch.Tensor],
    band_res: tuple[int, int, int],
    field_res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    *,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Inverse of :func:`roll_pad_partition_windows_band`: the band's tokens ``(B, C, H_band, W, D)``;
    its first ``s`` rows are read from ``halo_in`` (the previous band's :func:`band_halo_extract`)."""
    if windows.device.type != "cuda" or windows.dtype not in _DTYPES:
        raise ValueError("crop_roll_unmerge_windows_band requires CUDA float32/bfloat16 windows.")
    out_dtype = windows.dtype if out_dtype is None else out_dtype
    if out_dtype not in _DTYPES:
        raise ValueError("out_dtype must be float32 or bfloat16")
    C, Hb, W = (int(v) for v in band_res)
    ws, ss, nW, N = band_geometry(band_res, field_res, window_size, shift_size)
    BnW, Nw, D = windows.shape
    if BnW % nW or Nw != N:
        raise ValueError(f"windows {tuple(windows.shape)} do not match the band's {nW} windows of {N} tokens")
    B = BnW // nW
    halo_in = _check_halo(halo_in, B, C, ss[1], W, D, windows.dtype, windows.device, "halo_in")
    windows = windows.contiguous()
    out = torch.empty((B, C, Hb, W, D), device=windows.device, dtype=out_dtype)
    rc = _lib.load().fa_crop_roll_unmerge_band(
        windows.data_ptr(), halo_in.data_ptr() if halo_in is not None else None, _lib.dtype_code(windows.dtype),
        out.data_ptr(), _lib.dtype_code(out_dtype), B, C, Hb, field_res[1], W, D,
        _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.stream_ptr(windows.device))
    _lib.check(rc, "crop_roll_unmerge_windows_band")
    return out
