"""Shifted-window attention (N <= 144 tokens per window, head_dim 64) on the B200 kernels.

Drop-in for upstream ``flash_aurora/aurora/ops/cute/window_attn_fwd.py``: ``WinAttnPrecision``,
``window_attn_fwd_cute``, ``window_attn_fwd_cute_qkvpacked`` and ``window_attn_dispatch`` keep
their names, argument meaning and error behaviour (``AssertionError`` on a dtype/precision
mismatch, ``RuntimeError`` for non-CUDA tensors, ``ValueError``/``TypeError`` for bad shapes).
``tile_m``/``tile_n`` are accepted for signature compatibility; the B200 kernels pick their own
tiling.

Masks: a float ``bias (nW, N, N)`` is packed the upstream way (``bias < -50`` means masked,
``_window_softmax.py:151-153``) and a masked logit gets -100 after scaling. The block path
instead passes ``group_ids (nW, N)`` region ids (``shifted_window_group_ids``), which encode the
same Swin mask in N bytes per window instead of N*N.
"""

from __future__ import annotations

import ctypes
import math
from enum import Enum
from functools import lru_cache
from typing import Optional

import numpy as np
import torch

from . import _lib
from .recorder import KernelRecorder
from .util import window_geometry

__all__ = [
    "WinAttnPrecision",
    "window_attn_fwd_cute",
    "window_attn_fwd_cute_qkvpacked",
    "window_attn_dispatch",
    "shifted_window_group_ids",
    "swin_attn_mask_u8",
]

WINDOW_ATTN_MASK_THRESHOLD = -50.0


# Optional launch recorder for benchmarks: when installed with set_recorder, every packed-QKV
# attention launch is bracketed by CUDA events on its stream, with its algorithmic bytes and FLOPs
# (Q, K, V read + O written; 4 * Bwin * H * N^2 * Dh FLOPs).
_RECORDER: Optional[KernelRecorder] = None


def set_recorder(rec: Optional[KernelRecorder]) -> None:
    global _RECORDER
    _RECORDER = rec


def _record_begin():
    if _RECORDER is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


def _record_end(ev0, Bwin, H, N, Dh, elem_bytes):
    if ev0 is None or _RECORDER is None:
        return
    ev1 = torch.cuda.Event(enable_timing=True)
    ev1.record()
    _RECORDER.records.append((ev0, ev1, 4 * Bwin * H * N * Dh * elem_bytes, 4 * Bwin * H * N * N * Dh))


class WinAttnPrecision(Enum):
    """Precision of :func:`window_attn_fwd_cute` (upstream window_attn_fwd.py:49-60).

    ``BF16_MIXED``     bf16 I/O, fp32 accumulation and softmax.
    ``TF32_ACC_FP32``  fp32 I/O. Here computed with 3xTF32 split products (fp32-level accuracy);
                       the upstream kernel uses 1xTF32 QK^T and bf16 P.V.
    """

    BF16_MIXED = "bf16_mixed"
    TF32_ACC_FP32 = "tf32_acc_fp32"


def swin_attn_mask_u8(bias: torch.Tensor) -> torch.Tensor:
    """Pack a float Swin bias ``(nW, N, N)`` into a uint8 mask (1 = masked)."""
    return (bias < WINDOW_ATTN_MASK_THRESHOLD).to(torch.uint8).contiguous()


@lru_cache(maxsize=64)
def _group_ids_host(res, window_size, shift_size, warped):
    _, _, _, _, nW, N = window_geometry(tuple(res), tuple(window_size), tuple(shift_size))
    buf = np.empty((nW, N), dtype=np.uint8)
    rc = _lib.load().fa_shifted_window_groups(
        int(res[0]), int(res[1]), int(res[2]), _lib.i32x3(window_size), _lib.i32x3(shift_size),
        int(bool(warped)), buf.ctypes.data_as(ctypes.c_void_p))
    _lib.check(rc, "shifted_window_group_ids")
    buf.setflags(write=False)
    return buf


_GROUP_CACHE: dict = {}
# Attribute set on region-id tensors known to fit the tensor-core mask: every window has at most
# 16 distinct ids, all below 32 (FA_ATTN_FLAG_REGIONS_FIT).
_REGIONS_FIT = "_fa_regions_fit"


def region_ids_fit(ids: np.ndarray) -> bool:
    """True when every window (row) of ``ids`` has at most 16 distinct values, all below 32."""
    ids = np.asarray(ids)
    if ids.size == 0:
        return True
    if int(ids.max()) >= 32:
        return False
    present = np.zeros((ids.shape[0], 32), dtype=bool)
    present[np.arange(ids.shape[0])[:, None], ids.astype(np.int64)] = True
    return bool((present.sum(axis=1) <= 16).all())


def mark_region_ids_fit(t: torch.Tensor, fits: bool = True) -> torch.Tensor:
    """Record on ``t`` that its region ids fit the tensor-core mask (see :func:`region_ids_fit`)."""
    setattr(t, _REGIONS_FIT, bool(fits))
    return t


def shifted_window_group_ids(res, window_size, shift_size, warped: bool = True,
                             device: Optional[torch.device] = None) -> torch.Tensor:
    """``(nW, N)`` uint8 region ids of the shifted-window mask (upstream swin3d.py:526-599)."""
    key = (tuple(res), tuple(window_size), tuple(shift_size), bool(warped), str(device))
    t = _GROUP_CACHE.get(key)
    if t is None:
        arr = _group_ids_host(tuple(res), tuple(window_size), tuple(shift_size), bool(warped))
        host = torch.from_numpy(arr.copy())
        t = host.to(device) if device is not None else host
        mark_region_ids_fit(t, region_ids_fit(arr))
        _GROUP_CACHE[key] = t
    return t


def _attn_flags(group_ids: Optional[torch.Tensor]) -> int:
    if group_ids is not None and getattr(group_ids, _REGIONS_FIT, False):
        return _lib.FA_ATTN_FLAG_REGIONS_FIT
    return 0


def _precision_code(precision: WinAttnPrecision) -> int:
    return _lib.FA_ATTN_FP32_3XTF32 if precision == WinAttnPrecision.TF32_ACC_FP32 else _lib.FA_ATTN_BF16


def _require_cuda(t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError("B200 window attention requires CUDA tensors.")


def _mask_args(bias, group_ids, device, N):
    mask_u8 = None
    if bias is not None:
        if bias.ndim != 3 or bias.shape[1] != N or bias.shape[2] != N:
            raise ValueError(f"bias must have shape (nW, {N}, {N}), got {tuple(bias.shape)}")
        mask_u8 = swin_attn_mask_u8(bias.to(device))
        return mask_u8, None, int(bias.shape[0]), mask_u8
    if group_ids is not None:
        if group_ids.ndim != 2 or group_ids.shape[1] != N or group_ids.dtype != torch.uint8:
            raise ValueError(f"group_ids must be uint8 (nW, {N}), got {tuple(group_ids.shape)} {group_ids.dtype}")
        g = group_ids.to(device).contiguous()
        return None, g, int(g.shape[0]), g
    return None, None, 0, None


def window_attn_fwd_cute(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    scale_qk: Optional[float] = None,
    precision: WinAttnPrecision = WinAttnPrecision.BF16_MIXED,
    tile_m: int = 64,
    tile_n: Optional[int] = None,
    group_ids: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Attention on ``q, k, v (Bwin, H, N, Dh)`` with an optional per-window mask
    (upstream window_attn_fwd.py:141-243). Returns ``(Bwin, H, N, Dh)``."""
    if precision == WinAttnPrecision.TF32_ACC_FP32:
        assert q.dtype == torch.float32, "TF32_ACC_FP32 requires float32 tensors"
    else:
        assert q.dtype == torch.bfloat16, "BF16_MIXED requires bfloat16 tensors"
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share a dtype")
    if q.shape != k.shape or q.shape != v.shape or q.ndim != 4:
        raise ValueError("q, k, v must all be (Bwin, H, N, Dh)")
    _require_cuda(q)
    Bwin, H, N, Dh = q.shape
    if scale_qk is None:
        scale_qk = 1.0 / math.sqrt(Dh)
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    mask_u8, gids, nW, keep = _mask_args(bias, group_ids, q.device, N)
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])
    rc = _lib.load().fa_window_attention(
        _precision_code(precision), Bwin, H, N, Dh, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
        strides, mask_u8.data_ptr() if mask_u8 is not None else None,
        gids.data_ptr() if gids is not None else None, nW, float(scale_qk), _attn_flags(group_ids),
        _lib.stream_ptr(q.device))
    _lib.check(rc, "window_attn_fwd_cute")
    del keep
    return out


def window_attn_fwd_cute_qkvpacked(
    qkv: torch.Tensor,
    num_heads: int,
    bias: Optional[torch.Tensor] = None,
    *,
    scale_qk: Optional[float] = None,
    tile_m: Optional[int] = None,
    tile_n: Optional[int] = None,
    output_layout: str = "bhnd",
    group_ids: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Attention reading Q/K/V straight from the packed ``Linear(D, 3D)`` output
    ``(Bwin, N, 3 * H * Dh)`` (upstream window_attn_fwd.py:246-353). Precision follows the dtype."""
    if qkv.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"qkv-packed path supports bfloat16 and float32; got {qkv.dtype}")
    if qkv.ndim != 3:
        raise ValueError(f"qkv must have shape (Bwin, N, 3*C); got {tuple(qkv.shape)}")
    if not qkv.is_contiguous():
        raise ValueError("qkv-packed path requires contiguous qkv linear output")
    if qkv.shape[-1] % (3 * num_heads) != 0:
        raise ValueError(f"last dim {qkv.shape[-1]} must be divisible by 3*num_heads={3 * num_heads}")
    if output_layout not in {"bhnd", "bnc"}:
        raise ValueError(f"output_layout must be 'bhnd' or 'bnc', got {output_layout!r}")
    _require_cuda(qkv)
    Bwin, N, three_c = qkv.shape
    H = num_heads
    Dh = three_c // (3 * H)
    if scale_qk is None:
        scale_qk = 1.0 / math.sqrt(Dh)
    shape = (Bwin, N, H * Dh) if output_layout == "bnc" else (Bwin, H, N, Dh)
    if out is None:
        out = torch.empty(shape, device=qkv.device, dtype=qkv.dtype)
    elif tuple(out.shape) != shape or out.dtype != qkv.dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {qkv.dtype} tensor of shape {shape}")
    mask_u8, gids, nW, keep = _mask_args(bias, group_ids, qkv.device, N)
    prec = _lib.FA_ATTN_BF16 if qkv.dtype == torch.bfloat16 else _lib.FA_ATTN_FP32_3XTF32
    layout = _lib.FA_LAYOUT_BNC if output_layout == "bnc" else _lib.FA_LAYOUT_BHND
    ev0 = _record_begin()
    rc = _lib.load().fa_window_attention_qkvpacked(
        prec, Bwin, N, H, Dh, qkv.data_ptr(), out.data_ptr(), layout,
        mask_u8.data_ptr() if mask_u8 is not None else None, gids.data_ptr() if gids is not None else None,
        nW, float(scale_qk), _attn_flags(group_ids), _lib.stream_ptr(qkv.device))
    _lib.check(rc, "window_attn_fwd_cute_qkvpacked")
    _record_end(ev0, Bwin, H, N, Dh, qkv.element_size())
    del keep
    return out


def window_attn_dispatch(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    scale_qk: Optional[float] = None,
    tile_m: int = 64,
    tile_n: Optional[int] = None,
) -> torch.Tensor:
    """Precision from ``q.dtype`` (upstream window_attn_fwd.py:360-394)."""
    precision = WinAttnPrecision.BF16_MIXED if q.dtype == torch.bfloat16 else WinAttnPrecision.TF32_ACC_FP32
    return window_attn_fwd_cute(q, k, v, bias, scale_qk=scale_qk, precision=precision, tile_m=tile_m, tile_n=tile_n)
