"""C ABI checks that need no GPU: the library loads, exports every declared symbol, and its
host-only entry points (geometry, shifted-window region ids, argument validation) match the
oracle and the upstream fixtures."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from oracle import layout as OL

HEADER = os.path.join(ROOT, "include", "flash_aurora_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from flash_aurora_b200 import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from flash_aurora_b200 import _lib
    names = _declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.fa_version() >= 100


def test_geometry_matches_oracle(lib, golden):
    from flash_aurora_b200.util import window_geometry
    d = golden("layout_maps.npz")
    for name in sorted({k.split("/")[0] for k in d if k.endswith("/spec")}):
        spec = d[f"{name}/spec"]
        res, ws, ss = tuple(spec[:3]), tuple(spec[3:6]), tuple(spec[6:9])
        g = OL.geometry(res, ws, ss)
        got = window_geometry(tuple(int(a) for a in res), tuple(int(a) for a in ws), tuple(int(a) for a in ss))
        assert got == (g.ws, g.ss, g.pad_front, g.padded, g.num_windows, g.window_tokens), name


def test_region_ids_match_upstream(lib, golden):
    from flash_aurora_b200.window_attn import _group_ids_host
    d = golden("mask_groups.npz")
    for name in sorted({k.split("/")[0] for k in d if k.endswith("/spec")}):
        spec = [int(a) for a in d[f"{name}/spec"]]
        got = _group_ids_host(tuple(spec[:3]), tuple(spec[3:6]), tuple(spec[6:9]), bool(spec[9]))
        np.testing.assert_array_equal(got, d[f"{name}/groups"], err_msg=name)


def test_region_ids_on_the_shape_upstream_rejects(lib):
    # Upstream compute_3d_shifted_window_mask raises at this shape (a 1 x 1 x W window grid);
    # the restated algorithm still defines the ids and both implementations agree.
    from flash_aurora_b200.window_attn import _group_ids_host
    got = _group_ids_host((2, 5, 30), (2, 6, 12), (1, 3, 6), True)
    np.testing.assert_array_equal(got, OL.window_group_ids((2, 5, 30), (2, 6, 12), (1, 3, 6)))


def test_invalid_arguments_return_status_without_a_gpu(lib):
    from flash_aurora_b200 import _lib
    ws, ss = _lib.i32x3((2, 6, 12)), _lib.i32x3((1, 3, 6))
    rc = lib.fa_roll_pad_partition(None, 0, None, 0, 1, 4, 36, 72, 256, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"null" in lib.fa_last_error()
    rc = lib.fa_roll_pad_partition(ctypes.c_void_p(16), 7, ctypes.c_void_p(16), 0, 1, 4, 36, 72, 256, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"dtype" in lib.fa_last_error()
    rc = lib.fa_crop_roll_unmerge(ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, 1, 0, 36, 72, 256, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID
    strides = (ctypes.c_int64 * 12)(*([64] * 12))
    p = ctypes.c_void_p(1 << 20)
    rc = lib.fa_window_attention(0, 4, 8, 144, 32, p, p, p, p, strides, None, None, 0, 0.125, 0, None)
    assert rc == _lib.FA_ERR_UNSUPPORTED and b"head_dim" in lib.fa_last_error()
    rc = lib.fa_window_attention(0, 4, 8, 288, 64, p, p, p, p, strides, None, None, 0, 0.125, 0, None)
    assert rc == _lib.FA_ERR_UNSUPPORTED
    rc = lib.fa_window_attention(5, 4, 8, 144, 64, p, p, p, p, strides, None, None, 0, 0.125, 0, None)
    assert rc == _lib.FA_ERR_INVALID
    rc = lib.fa_adaln_film(p, 0, None, 0, p, p, 0, 0.0, 1e-5, p, 0, None, 1, 4, 4096, None)
    assert rc == _lib.FA_ERR_UNSUPPORTED and b"2048" in lib.fa_last_error()
    rc = lib.fa_adaln_film(p, 0, p, 1, p, p, 0, 0.0, 1e-5, p, 0, None, 1, 4, 256, None)
    assert rc == _lib.FA_ERR_INVALID and b"residual" in lib.fa_last_error()


def test_band_arguments_return_status_without_a_gpu(lib):
    from flash_aurora_b200 import _lib
    ws, ss = _lib.i32x3((2, 6, 12)), _lib.i32x3((1, 3, 6))
    p = ctypes.c_void_p(1 << 20)
    # band height not a whole number of window rows
    rc = lib.fa_roll_pad_partition_band(p, p, 0, 0, p, 0, 1, 4, 9, 36, 72, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"band height" in lib.fa_last_error()
    # field height needing padding along H
    rc = lib.fa_roll_pad_partition_band(p, p, 0, 0, p, 0, 1, 4, 6, 45, 90, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_UNSUPPORTED and b"multiple of the window height" in lib.fa_last_error()
    # shifted band without its halo
    rc = lib.fa_roll_pad_partition_band(p, None, 0, 0, p, 0, 1, 4, 12, 36, 72, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"halo" in lib.fa_last_error()
    # a halo in neither the input's nor the windows' dtype
    rc = lib.fa_roll_pad_partition_band(p, p, 0, 1, p, 0, 1, 4, 12, 36, 72, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"halo_dtype" in lib.fa_last_error()
    rc = lib.fa_crop_roll_unmerge_band(p, None, 0, p, 0, 1, 4, 12, 36, 72, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID and b"halo" in lib.fa_last_error()
    rc = lib.fa_unmerge_adaln_film_band(p, None, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None,
                                        1, 4, 12, 36, 72, 64, ws, ss, 0, 12, None)
    assert rc == _lib.FA_ERR_INVALID and b"halo" in lib.fa_last_error()
    # rows that start below the halo depth (s = 3) still need it
    rc = lib.fa_unmerge_adaln_film_band(p, None, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None,
                                        1, 4, 12, 36, 72, 64, ws, ss, 2, 10, None)
    assert rc == _lib.FA_ERR_INVALID and b"halo" in lib.fa_last_error()
    # row ranges past the band, and an empty range (nothing launched)
    rc = lib.fa_unmerge_adaln_film_band(p, p, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None,
                                        1, 4, 12, 36, 72, 64, ws, ss, 6, 7, None)
    assert rc == _lib.FA_ERR_INVALID and b"row range" in lib.fa_last_error()
    assert lib.fa_unmerge_adaln_film_band(p, None, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None,
                                          1, 4, 12, 36, 72, 64, ws, ss, 3, 0, None) == _lib.FA_OK
    rc = lib.fa_adaln_film_rows(p, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None, 1, 4, 12, 72, 64, -1, 2, None)
    assert rc == _lib.FA_ERR_INVALID and b"row range" in lib.fa_last_error()
    rc = lib.fa_adaln_film_rows(p, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None, 1, 4, 12, 72, 64, 10, 3, None)
    assert rc == _lib.FA_ERR_INVALID and b"row range" in lib.fa_last_error()
    assert lib.fa_adaln_film_rows(p, 0, p, 0, p, p, 0, 0.0, 1e-5, p, 0, None, 1, 4, 12, 72, 64, 5, 0,
                                  None) == _lib.FA_OK
    # band taller than the field
    rc = lib.fa_band_halo_extract(p, 0, p, 0, 1, 4, 42, 36, 72, 64, ws, ss, None)
    assert rc == _lib.FA_ERR_INVALID
    # an unshifted band needs no halo and nothing is extracted (no launch, so no GPU needed)
    z = _lib.i32x3((0, 0, 0))
    assert lib.fa_band_halo_extract(p, 0, p, 0, 1, 4, 12, 36, 72, 64, ws, z, None) == _lib.FA_OK


def test_attention_flags_validated_without_a_gpu(lib):
    from flash_aurora_b200 import _lib
    strides = (ctypes.c_int64 * 12)(*([64] * 12))
    p = ctypes.c_void_p(1 << 20)
    rc = lib.fa_window_attention(0, 4, 8, 144, 64, p, p, p, p, strides, None, None, 0, 0.125, 6, None)
    assert rc == _lib.FA_ERR_INVALID and b"flags" in lib.fa_last_error()


def test_region_ids_fit_rule():
    from flash_aurora_b200.window_attn import region_ids_fit
    assert region_ids_fit(OL.window_group_ids((4, 36, 72), (2, 6, 12), (1, 3, 6)))
    assert region_ids_fit(OL.window_group_ids((4, 45, 90), (2, 6, 12), (1, 3, 6)))
    assert region_ids_fit(np.tile(np.arange(16, dtype=np.uint8), (3, 9)))
    assert not region_ids_fit(np.tile(np.arange(17, dtype=np.uint8), (2, 1)))
    assert not region_ids_fit(np.full((2, 144), 40, dtype=np.uint8))


def test_layernorm_arguments_return_status_without_a_gpu(lib):
    from flash_aurora_b200 import _lib
    p = ctypes.c_void_p(1 << 20)
    rc = lib.fa_layernorm_affine(p, 3, None, p, p, 0, 1e-5, p, 4, 256, None)
    assert rc == _lib.FA_ERR_INVALID and b"dtype" in lib.fa_last_error()
    rc = lib.fa_layernorm_affine(p, 0, None, p, p, 0, 1e-5, p, 4, 4097, None)
    assert rc == _lib.FA_ERR_UNSUPPORTED and b"4096" in lib.fa_last_error()
    rc = lib.fa_layernorm_affine(None, 0, None, p, p, 0, 1e-5, p, 4, 256, None)
    assert rc == _lib.FA_ERR_INVALID and b"null" in lib.fa_last_error()
    assert lib.fa_layernorm_affine(None, 0, None, None, None, 0, 1e-5, None, 0, 256, None) == _lib.FA_OK


def test_perceiver_ln_shim_rejects_like_upstream():
    import torch
    import flash_aurora_b200 as fa
    x = torch.zeros(2, 3, 8)
    with pytest.raises(ValueError, match="CUDA"):
        fa.layernorm_affine_forward(x, torch.ones(8), torch.zeros(8), 1e-5)
    with pytest.raises(ValueError, match="residual"):
        fa.layernorm_affine_add_residual_forward(x, torch.zeros(2, 3, 9), torch.ones(8), torch.zeros(8), 1e-5)
