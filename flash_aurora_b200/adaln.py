"""Fused AdaLN (LayerNorm without affine + FiLM modulation) with optional residual add.

Drop-in for upstream ``flash_aurora/aurora/ops/triton_adaln.py``: same function names,
arguments, output dtypes and ``ValueError`` cases (CUDA, float32/bfloat16, ``D <= 2048``,
residual/x dtype rules, shapes). Extensions used by the block: ``out_bf16`` (a second, bfloat16
copy of the output for the next BF16 GEMM) and the unmerge-fused variant that reads the
AdaLN input straight from attention windows.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .util import band_geometry, window_geometry

__all__ = [
    "adaptive_layernorm_film_forward",
    "adaptive_layernorm_film_add_residual_forward",
    "unmerge_adaptive_layernorm_film_add_residual",
    "unmerge_adaptive_layernorm_film_add_residual_band",
    "adaptive_layernorm_film_add_residual_partition",
    "adaptive_layernorm_film_add_residual_rows",
]

_MAX_D = 2048
_DTYPES = (torch.float32, torch.bfloat16)


def _mod_rows(t: torch.Tensor, B: int, D: int, name: str) -> torch.Tensor:
    if tuple(t.shape) not in ((B, 1, D), (B, D)):
        raise ValueError(f"{name} must have shape (B, 1, D) = {(B, 1, D)}, got {tuple(t.shape)}")
    if t.dtype not in _DTYPES:
        raise ValueError(f"{name} must be float32 or bfloat16")
    return t.reshape(B, D).contiguous()


def _check_out_bf16(out_bf16: Optional[torch.Tensor], B: int, L: int, D: int, device) -> None:
    if out_bf16 is None:
        return
    if (tuple(out_bf16.shape) != (B, L, D) or out_bf16.dtype != torch.bfloat16
            or not out_bf16.is_contiguous() or out_bf16.device != device):
        raise ValueError(f"out_bf16 must be a contiguous bfloat16 tensor of shape {(B, L, D)} on {device}")


def _launch(x, residual, scale, shift, scale_bias, eps, out, out_bf16, B, L, D, what):
    rc = _lib.load().fa_adaln_film(
        x.data_ptr(), _lib.dtype_code(x.dtype),
        residual.data_ptr() if residual is not None else None,
        _lib.dtype_code(residual.dtype) if residual is not None else 0,
        scale.data_ptr(), shift.data_ptr(), _lib.dtype_code(scale.dtype),
        float(scale_bias), float(eps), out.data_ptr(), _lib.dtype_code(out.dtype),
        out_bf16.data_ptr() if out_bf16 is not None else None, B, L, D, _lib.stream_ptr(x.device))
    _lib.check(rc, what)


def adaptive_layernorm_film_forward(
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    scale_bias: float,
    eps: float = 1e-5,
    *,
    output_fp32: bool = False,
) -> torch.Tensor:
    """``LN(x) * (scale_bias + scale) + shift`` (upstream triton_adaln.py:33-80)."""
    if x.device.type != "cuda" or x.dtype not in _DTYPES:
        raise ValueError("adaptive_layernorm_film_forward requires CUDA float32/bfloat16 x.")
    B, L, D = x.shape
    if D > _MAX_D:
        raise ValueError(f"adaptive_layernorm_film_forward supports D <= {_MAX_D} for now.")
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    out = torch.empty(B, L, D, device=x.device, dtype=torch.float32 if output_fp32 else x.dtype)
    _launch(x.contiguous(), None, scale, shift, scale_bias, eps, out, None, B, L, D,
            "adaptive_layernorm_film_forward")
    return out


def adaptive_layernorm_film_add_residual_forward(
    residual: torch.Tensor,
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    scale_bias: float,
    eps: float = 1e-5,
    *,
    output_fp32: bool = False,
    out: Optional[torch.Tensor] = None,
    out_bf16: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``residual + LN(x) * (scale_bias + scale) + shift`` (upstream triton_adaln.py:83-145)."""
    if residual.device.type != "cuda" or x.device.type != "cuda":
        raise ValueError("adaptive_layernorm_film_add_residual_forward requires CUDA tensors.")
    if residual.dtype not in _DTYPES or x.dtype not in _DTYPES:
        raise ValueError("adaptive_layernorm_film_add_residual_forward requires float32/bfloat16.")
    if not output_fp32 and residual.dtype != x.dtype:
        raise ValueError("residual and x must have the same dtype unless output_fp32=True.")
    if output_fp32 and residual.dtype != torch.float32:
        raise ValueError("output_fp32=True requires residual.dtype == float32.")
    if residual.shape != x.shape:
        raise ValueError("residual and x must have the same shape.")
    B, L, D = x.shape
    if D > _MAX_D:
        raise ValueError(f"adaptive_layernorm_film_add_residual_forward supports D <= {_MAX_D}.")
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    out_dtype = torch.float32 if output_fp32 else x.dtype
    if out is None:
        out = torch.empty(B, L, D, device=x.device, dtype=out_dtype)
    elif (tuple(out.shape) != (B, L, D) or out.dtype != out_dtype or not out.is_contiguous()
          or out.device != x.device):
        raise ValueError(f"out must be a contiguous {out_dtype} tensor of shape {(B, L, D)} on {x.device}")
    _check_out_bf16(out_bf16, B, L, D, x.device)
    _launch(x.contiguous(), residual.contiguous(), scale, shift, scale_bias, eps, out, out_bf16, B, L, D,
            "adaptive_layernorm_film_add_residual_forward")
    return out


def adaptive_layernorm_film_add_residual_rows(
    residual: torch.Tensor,
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    res: tuple[int, int, int],
    rows: tuple[int, int],
    scale_bias: float,
    eps: float = 1e-5,
    *,
    out: torch.Tensor,
    out_bf16: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """:func:`adaptive_layernorm_film_add_residual_forward` (fp32 output) on the token rows
    ``(b, c, h, w)`` of the ``res = (C, H, W)`` grid with ``h`` in ``[rows[0], rows[0] + rows[1])``,
    written into ``out``; other rows of ``out`` are untouched. Two calls over complementary row
    ranges equal one full call."""
    for t in (residual, x, out):
        _lib.require_cuda(t, "adaptive_layernorm_film_add_residual_rows")
    if residual.dtype != torch.float32 or x.dtype not in _DTYPES:
        raise ValueError("residual must be float32 and x float32/bfloat16")
    if residual.shape != x.shape:
        raise ValueError("residual and x must have the same shape.")
    C, H, W = (int(v) for v in res)
    B, L, D = x.shape
    if L != C * H * W:
        raise ValueError(f"x has {L} tokens, res {tuple(res)} has {C * H * W}")
    if D > _MAX_D:
        raise ValueError(f"AdaLN supports D <= {_MAX_D}")
    h0, hn = int(rows[0]), int(rows[1])
    if h0 < 0 or hn < 0 or h0 + hn > H:
        raise ValueError(f"rows {rows} outside the grid's {H} rows")
    if (tuple(out.shape) != (B, L, D) or out.dtype != torch.float32 or not out.is_contiguous()
            or out.device != x.device):
        raise ValueError(f"out must be a contiguous float32 tensor of shape {(B, L, D)} on {x.device}")
    _check_out_bf16(out_bf16, B, L, D, x.device)
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    x, residual = x.contiguous(), residual.contiguous()
    rc = _lib.load().fa_adaln_film_rows(
        x.data_ptr(), _lib.dtype_code(x.dtype), residual.data_ptr(), _lib.FA_F32, scale.data_ptr(),
        shift.data_ptr(), _lib.dtype_code(scale.dtype), float(scale_bias), float(eps), out.data_ptr(),
        _lib.FA_F32, out_bf16.data_ptr() if out_bf16 is not None else None, B, C, H, W, D, h0, hn,
        _lib.stream_ptr(x.device))
    _lib.check(rc, "adaptive_layernorm_film_add_residual_rows")
    return out


def unmerge_adaptive_layernorm_film_add_residual(
    windows: torch.Tensor,
    residual: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    scale_bias: float = 0.0,
    eps: float = 1e-5,
    *,
    out_bf16: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``residual + AdaLN(crop_roll_unmerge(windows))`` in one pass, fp32 output.

    Replaces the upstream pair ``crop_roll_unmerge_windows_triton`` + ``norm1.forward_add_residual``
    (swin3d.py:751-800, film.py:101-139): the merged branch tensor is never materialised.
    """
    for t, n in ((windows, "windows"), (residual, "residual")):
        _lib.require_cuda(t, "unmerge_adaptive_layernorm_film_add_residual")
    if windows.dtype not in _DTYPES or residual.dtype != torch.float32:
        raise ValueError("windows must be float32/bfloat16 and residual float32")
    C, H, W = res
    B, L, D = residual.shape
    if L != C * H * W:
        raise ValueError(f"residual has {L} tokens, res {tuple(res)} has {C * H * W}")
    if D > _MAX_D:
        raise ValueError(f"AdaLN supports D <= {_MAX_D}")
    _, _, _, _, nW, N = window_geometry(tuple(res), tuple(window_size), tuple(shift_size))
    if tuple(windows.shape) != (B * nW, N, D):
        raise ValueError(f"windows must have shape {(B * nW, N, D)}, got {tuple(windows.shape)}")
    _check_out_bf16(out_bf16, B, L, D, residual.device)
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    out = torch.empty(B, L, D, device=residual.device, dtype=torch.float32)
    rc = _lib.load().fa_unmerge_adaln_film(
        windows.contiguous().data_ptr(), _lib.dtype_code(windows.dtype), residual.contiguous().data_ptr(),
        _lib.FA_F32, scale.data_ptr(), shift.data_ptr(), _lib.dtype_code(scale.dtype), float(scale_bias),
        float(eps), out.data_ptr(), _lib.FA_F32, out_bf16.data_ptr() if out_bf16 is not None else None,
        B, C, H, W, D, _lib.i32x3(window_size), _lib.i32x3(shift_size), _lib.stream_ptr(residual.device))
    _lib.check(rc, "unmerge_adaptive_layernorm_film_add_residual")
    return out


def unmerge_adaptive_layernorm_film_add_residual_band(
    windows: torch.Tensor,
    halo_in: Optional[torch.Tensor],
    residual: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    band_res: tuple[int, int, int],
    field_res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    scale_bias: float = 0.0,
    eps: float = 1e-5,
    *,
    out_bf16: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    rows: Optional[tuple[int, int]] = None,
) -> torch.Tensor:
    """Latitude-band form of :func:`unmerge_adaptive_layernorm_film_add_residual`: the band's first
    ``s = shift_h`` rows are read from ``halo_in (B, C, s, W, D)``, the previous band's halo
    extract (same dtype as ``windows``).

    ``rows = (h_begin, h_count)`` writes only those band rows of ``out`` (and ``out_bf16``);
    ``halo_in`` may then be ``None`` when ``h_begin >= s``. Used to normalise the rows that need
    no halo while the halo is in flight."""
    _lib.require_cuda(windows, "unmerge_adaptive_layernorm_film_add_residual_band")
    _lib.require_cuda(residual, "unmerge_adaptive_layernorm_film_add_residual_band")
    if windows.dtype not in _DTYPES or residual.dtype != torch.float32:
        raise ValueError("windows must be float32/bfloat16 and residual float32")
    C, Hb, W = (int(v) for v in band_res)
    B, L, D = residual.shape
    if L != C * Hb * W:
        raise ValueError(f"residual has {L} tokens, band {tuple(band_res)} has {C * Hb * W}")
    if D > _MAX_D:
        raise ValueError(f"AdaLN supports D <= {_MAX_D}")
    ws, ss, nW, N = band_geometry(band_res, field_res, window_size, shift_size)
    if tuple(windows.shape) != (B * nW, N, D):
        raise ValueError(f"windows must have shape {(B * nW, N, D)}, got {tuple(windows.shape)}")
    h0, hn = (0, Hb) if rows is None else (int(rows[0]), int(rows[1]))
    if h0 < 0 or hn < 0 or h0 + hn > Hb:
        raise ValueError(f"rows {rows} outside the band's {Hb} rows")
    if ss[1] and h0 < ss[1] and hn > 0:
        if halo_in is None:
            raise ValueError(f"a band with an H shift of {ss[1]} rows needs halo_in")
    if ss[1] and halo_in is not None:
        if tuple(halo_in.shape) != (B, C, ss[1], W, D) or halo_in.dtype != windows.dtype:
            raise ValueError(f"halo_in must be {windows.dtype} of shape {(B, C, ss[1], W, D)}")
        _lib.require_cuda(halo_in, "unmerge_adaptive_layernorm_film_add_residual_band")
        halo_in = halo_in.contiguous()
    else:
        halo_in = None
    _check_out_bf16(out_bf16, B, L, D, residual.device)
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    windows, residual = windows.contiguous(), residual.contiguous()
    if out is None:
        out = torch.empty(B, L, D, device=residual.device, dtype=torch.float32)
    elif (tuple(out.shape) != (B, L, D) or out.dtype != torch.float32 or not out.is_contiguous()
          or out.device != residual.device):
        raise ValueError(f"out must be a contiguous float32 tensor of shape {(B, L, D)} on {residual.device}")
    rc = _lib.load().fa_unmerge_adaln_film_band(
        windows.data_ptr(), halo_in.data_ptr() if halo_in is not None else None, _lib.dtype_code(windows.dtype),
        residual.data_ptr(), _lib.FA_F32, scale.data_ptr(), shift.data_ptr(), _lib.dtype_code(scale.dtype),
        float(scale_bias), float(eps), out.data_ptr(), _lib.FA_F32,
        out_bf16.data_ptr() if out_bf16 is not None else None, B, C, Hb, field_res[1], W, D,
        _lib.i32x3(window_size), _lib.i32x3(shift_size), h0, hn, _lib.stream_ptr(residual.device))
    _lib.check(rc, "unmerge_adaptive_layernorm_film_add_residual_band")
    return out


def adaptive_layernorm_film_add_residual_partition(
    residual: torch.Tensor,
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    res: tuple[int, int, int],
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    windows: torch.Tensor,
    scale_bias: float = 0.0,
    eps: float = 1e-5,
) -> torch.Tensor:
    """``out = residual + AdaLN(x)`` (fp32) that also writes ``out`` into ``windows`` in the layout
    of ``roll_pad_partition_windows(out, res, window_size, shift_size)`` (rounded to the windows'
    dtype): norm2 of one block fused with the partition of the next. Only token slots are written;
    ``windows`` must hold zeros in its pad slots (a zero-filled buffer reused across blocks)."""
    if residual.device.type != "cuda" or x.device.type != "cuda":
        raise ValueError("adaptive_layernorm_film_add_residual_partition requires CUDA tensors.")
    if residual.dtype != torch.float32 or x.dtype not in _DTYPES or residual.shape != x.shape:
        raise ValueError("residual must be float32 and x float32/bfloat16 of the same shape")
    C, H, W = (int(v) for v in res)
    B, L, D = x.shape
    if L != C * H * W:
        raise ValueError(f"x has {L} tokens, res {tuple(res)} has {C * H * W}")
    if D > _MAX_D:
        raise ValueError(f"AdaLN supports D <= {_MAX_D}")
    _, _, _, _, nW, N = window_geometry(tuple(res), tuple(window_size), tuple(shift_size))
    if (tuple(windows.shape) != (B * nW, N, D) or windows.dtype not in _DTYPES or not windows.is_contiguous()
            or windows.device != x.device):
        raise ValueError(f"windows must be a contiguous float32/bfloat16 tensor of shape {(B * nW, N, D)}")
    scale = _mod_rows(scale, B, D, "scale")
    shift = _mod_rows(shift, B, D, "shift").to(scale.dtype)
    x, residual = x.contiguous(), residual.contiguous()
    out = torch.empty(B, L, D, device=x.device, dtype=torch.float32)
    rc = _lib.load().fa_adaln_film_partition(
        x.data_ptr(), _lib.dtype_code(x.dtype), residual.data_ptr(), _lib.FA_F32, scale.data_ptr(),
        shift.data_ptr(), _lib.dtype_code(scale.dtype), float(scale_bias), float(eps), out.data_ptr(), _lib.FA_F32,
        windows.data_ptr(), _lib.dtype_code(windows.dtype), B, C, H, W, D, _lib.i32x3(window_size),
        _lib.i32x3(shift_size), _lib.stream_ptr(x.device))
    _lib.check(rc, "adaptive_layernorm_film_add_residual_partition")
    return out
