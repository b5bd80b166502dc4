"""ctypes binding of the in-tree CUDA library ``libflash_aurora_b200.so`` (C ABI in
``include/flash_aurora_b200.h``).

The library is the only compute path of this package: when it is missing, every op raises
``RuntimeError`` instead of falling back to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflash_aurora_b200.so")

FA_F32, FA_BF16, FA_F16 = 0, 1, 2
FA_OK, FA_ERR_INVALID, FA_ERR_UNSUPPORTED, FA_ERR_CUDA, FA_ERR_TIMEOUT = 0, -1, -2, -3, -4
FA_ATTN_BF16, FA_ATTN_FP32_3XTF32 = 0, 1
FA_LAYOUT_BHND, FA_LAYOUT_BNC = 0, 1
FA_GELU_ERFF, FA_GELU_POLY = 0, 1
FA_ATTN_FLAG_REGIONS_FIT = 1
FA_ACT_NONE, FA_ACT_GELU = 0, 1
FA_STATUS_REGIONS_BROKEN, FA_STATUS_WATCHDOG_SELFTEST = 28, 90
FA_ROWS_TOKENS, FA_ROWS_WINDOWS = 0, 1

_i64, _i32, _f32, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p
_u32 = ctypes.c_uint
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.c_void_p

# name -> (restype, argtypes); every symbol declared in include/flash_aurora_b200.h
SIGNATURES = {
    "fa_last_error": (ctypes.c_char_p, []),
    "fa_version": (_i32, []),
    "fa_window_geometry": (_i32, [_i64, _i64, _i64, _i32p, _i32p, _i32p, _i32p, _i32p, _i64p, _i64p, _i32p]),
    "fa_roll_pad_partition": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _vp]),
    "fa_crop_roll_unmerge": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _vp]),
    "fa_adaln_film": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _f32, _f32, _vp, _i32, _vp, _i64, _i64, _i64, _vp]),
    "fa_adaln_film_partition": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _f32, _f32, _vp, _i32, _vp, _i32,
                                       _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _vp]),
    "fa_unmerge_adaln_film": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _f32, _f32, _vp, _i32, _vp,
                                     _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _vp]),
    "fa_roll_pad_partition_band": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                          _i32p, _i32p, _vp]),
    "fa_band_halo_extract": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _vp]),
    "fa_crop_roll_unmerge_band": (_i32, [_vp, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                         _i32p, _i32p, _vp]),
    "fa_unmerge_adaln_film_band": (_i32, [_vp, _vp, _i32, _vp, _i32, _vp, _vp, _i32, _f32, _f32, _vp, _i32, _vp,
                                          _i64, _i64, _i64, _i64, _i64, _i64, _i32p, _i32p, _i64, _i64, _vp]),
    "fa_adaln_film_rows": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _f32, _f32, _vp, _i32, _vp, _i64, _i64, _i64,
                                  _i64, _i64, _i64, _i64, _vp]),
    "fa_linear_bias_act": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "fa_gemm_status": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "fa_gemm_status_reset": (_i32, [_vp]),
    "fa_patch_merge_ln": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp]),
    "fa_patch_split_ln": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32p, _f32, _vp]),
    "fa_gelu_erf": (_i32, [_vp, _vp, _i32, _i64, _i32, _vp]),
    "fa_shifted_window_groups": (_i32, [_i64, _i64, _i64, _i32p, _i32p, _i32, _u8p]),
    "fa_window_attention": (_i32, [_i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64p, _u8p, _u8p, _i64, _f32,
                                   _u32, _vp]),
    "fa_window_attention_qkvpacked": (_i32, [_i32, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _u8p, _u8p, _i64, _f32,
                                             _u32, _vp]),
    "fa_window_attention_bias_noalloc": (_i32, [_i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64p, _vp,
                                                 _i64, _f32, _vp]),
    "fa_layernorm_affine": (_i32, [_vp, _i32, _vp, _vp, _vp, _i32, _f32, _vp, _i64, _i64, _vp]),
    "fa_attention_status": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "fa_attention_status_reset": (_i32, [_vp]),
    "fa_watchdog_selftest": (_i32, [_i64, _vp]),
    "fa_linear_adaln_film": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _f32, _f32, _vp, _vp, _vp, _vp,
                                    _i64, _i64, _i64, _i64, _i32p, _i32p, _i32p, _vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the library once (raises ``RuntimeError`` when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"flash_aurora_b200 CUDA library not found at {LIB_PATH}; "
                    "build it with `python -m flash_aurora_b200.build`"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Map a C-ABI status to the exception types the upstream Python ops raise."""
    if rc == FA_OK:
        return
    msg = load().fa_last_error().decode(errors="replace")
    if rc in (FA_ERR_INVALID, FA_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {rc})")


def i32x3(v) -> ctypes.Array:
    return (ctypes.c_int32 * 3)(*[int(a) for a in v])


def dtype_code(t: torch.dtype) -> int:
    if t == torch.float32:
        return FA_F32
    if t == torch.bfloat16:
        return FA_BF16
    raise ValueError(f"unsupported dtype {t}; expected float32 or bfloat16")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} requires CUDA tensors (got {t.device})")
