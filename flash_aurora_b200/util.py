"""Window helpers shared by the ops (same behaviour as upstream ``aurora/model/util.py``)."""

from __future__ import annotations

import ctypes
from functools import lru_cache

from . import _lib

__all__ = ["maybe_adjust_windows", "window_geometry", "band_geometry"]


def maybe_adjust_windows(window_size, shift_size, res):
    """Clamp the window to the resolution and drop the shift on that axis
    (upstream ``flash_aurora/aurora/model/util.py:54-72``)."""
    assert len(window_size) == len(shift_size) == len(res)
    ws, ss = list(window_size), list(shift_size)
    for i in range(len(res)):
        if res[i] <= window_size[i]:
            ss[i] = 0
            ws[i] = res[i]
    assert min(ws) > 0, f"Window size must be positive. Found {tuple(ws)}."
    assert min(ss) >= 0, f"Shift size must be non-negative. Found {tuple(ss)}."
    return tuple(ws), tuple(ss)


@lru_cache(maxsize=256)
def window_geometry(res, window_size, shift_size):
    """Geometry from the C ABI: ``(ws, ss, pad_front, padded, num_windows, window_tokens)``."""
    lib = _lib.load()
    ws = (ctypes.c_int32 * 3)()
    ss = (ctypes.c_int32 * 3)()
    pf = (ctypes.c_int32 * 3)()
    padded = (ctypes.c_int64 * 3)()
    nw = ctypes.c_int64()
    n = ctypes.c_int32()
    rc = lib.fa_window_geometry(int(res[0]), int(res[1]), int(res[2]), _lib.i32x3(window_size),
                                _lib.i32x3(shift_size), ws, ss, pf, padded, ctypes.byref(nw),
                                ctypes.byref(n))
    _lib.check(rc, "window_geometry")
    return tuple(ws), tuple(ss), tuple(pf), tuple(padded), int(nw.value), int(n.value)


def band_geometry(band_res, field_res, window_size, shift_size):
    """``(ws, ss, num_windows, window_tokens)`` of a latitude band ``(C, H_band, W)`` of the field
    ``(C, H, W)``. Window clamping and shifts are decided on the field (as the unsharded block
    does); the band must hold whole window rows and the field must need no H padding."""
    band_res, field_res = tuple(int(v) for v in band_res), tuple(int(v) for v in field_res)
    ws, ss, pf, padded, nW, N = window_geometry(field_res, tuple(window_size), tuple(shift_size))
    C, Hb, W = band_res
    if (C, W) != (field_res[0], field_res[2]):
        raise ValueError(f"band {band_res} must share C and W with the field {field_res}")
    H = field_res[1]
    if padded[1] != H:
        raise ValueError(f"band sharding needs H ({H}) to be a multiple of the window height ({ws[1]})")
    if Hb <= 0 or Hb > H or Hb % ws[1]:
        raise ValueError(f"band height {Hb} must be a positive multiple of {ws[1]}, at most {H}")
    if ss[1] > Hb:
        raise ValueError(f"halo of {ss[1]} rows is deeper than the band ({Hb} rows)")
    return ws, ss, nW // (H // ws[1]) * (Hb // ws[1]), N
