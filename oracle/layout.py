"""numpy restatement of the Swin3D window layout and shifted-window mask (test oracle).

All functions here do integer/index work only and are compared bit-exactly.

Upstream semantics restated (paths relative to the Flash-Aurora project):

* ``maybe_adjust_windows``            flash_aurora/aurora/model/util.py:54-72
* three-sided symmetric zero padding  flash_aurora/aurora/model/swin3d.py:415-432,488-507
                                      (same split in ops/triton_swin3d_layout.py:27-55)
* roll(-ss) -> pad -> partition       flash_aurora/aurora/model/swin3d.py:757-770, 436-451;
                                      kernel ops/triton_swin3d_layout.py:192-250
* window merge -> crop -> roll(+ss)   flash_aurora/aurora/model/swin3d.py:775-789, 454-485;
                                      kernel ops/triton_swin3d_layout.py:253-307
* shifted-window mask groups          flash_aurora/aurora/model/swin3d.py:526-599

Latitude bands (a field split along H across ranks) have no upstream counterpart; the band
functions below restate them from the field definitions above by explicit concatenation, an
independent formulation of the index encoding used by the CUDA band kernels.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass

import numpy as np

# Upstream masks use a finite additive -100 after scaling (swin3d.py:597).
MASKED_BIAS = -100.0


def maybe_adjust_windows(window_size, shift_size, res):
    """util.py:54-72: clamp the window to the resolution and drop the shift on that axis."""
    ws, ss = list(window_size), list(shift_size)
    for i in range(len(res)):
        if res[i] <= window_size[i]:
            ss[i] = 0
            ws[i] = res[i]
    assert min(ws) > 0 and min(ss) >= 0
    return tuple(ws), tuple(ss)


def _split(p: int) -> tuple[int, int]:
    """swin3d.py:420-430: ``front = p // 2``, ``back = p - front`` (zero when ``p == 0``)."""
    if p:
        return p // 2, p - p // 2
    return 0, 0


@dataclass(frozen=True)
class Geometry:
    """Window geometry of one block call (triton_swin3d_layout.py:78-88)."""

    C: int
    H: int
    W: int
    ws: tuple[int, int, int]
    ss: tuple[int, int, int]
    pad_front: tuple[int, int, int]  # (front along C, top along H, left along W)
    padded: tuple[int, int, int]
    grid: tuple[int, int, int]  # windows per axis (C1, H1, W1)

    @property
    def num_windows(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def window_tokens(self) -> int:
        return self.ws[0] * self.ws[1] * self.ws[2]


def geometry(res, window_size, shift_size) -> Geometry:
    C, H, W = res
    ws, ss = maybe_adjust_windows(tuple(window_size), tuple(shift_size), tuple(res))
    pads = ((-C) % ws[0], (-H) % ws[1], (-W) % ws[2])
    fronts = tuple(_split(p)[0] for p in pads)
    padded = (C + pads[0], H + pads[1], W + pads[2])
    grid = tuple(padded[i] // ws[i] for i in range(3))
    return Geometry(C, H, W, ws, ss, fronts, padded, grid)


def partition_source_index(g: Geometry) -> np.ndarray:
    """Flat token index ``(c*H + h)*W + w`` feeding each ``(window, token)`` slot, or -1 (pad).

    Restates triton_swin3d_layout.py:218-246 for one batch element: window ``(c1, h1, w1)``
    with ``w1`` fastest, token ``(wc, wh, ww)`` with ``ww`` fastest; the padded position maps
    to the shifted position by subtracting the front pad and to the source by ``+ss mod dim``.
    """
    C, H, W = g.C, g.H, g.W
    Wc, Wh, Ww = g.ws
    C1, H1, W1 = g.grid
    c1, h1, w1, wc, wh, ww = np.meshgrid(
        np.arange(C1), np.arange(H1), np.arange(W1),
        np.arange(Wc), np.arange(Wh), np.arange(Ww), indexing="ij",
    )
    cs = c1 * Wc + wc - g.pad_front[0]
    hs = h1 * Wh + wh - g.pad_front[1]
    wsh = w1 * Ww + ww - g.pad_front[2]
    inside = (cs >= 0) & (cs < C) & (hs >= 0) & (hs < H) & (wsh >= 0) & (wsh < W)
    xc = np.mod(cs + g.ss[0], C)
    xh = np.mod(hs + g.ss[1], H)
    xw = np.mod(wsh + g.ss[2], W)
    src = (xc * H + xh) * W + xw
    src = np.where(inside, src, -1)
    return src.reshape(g.num_windows, g.window_tokens).astype(np.int64)


def unmerge_source_index(g: Geometry) -> np.ndarray:
    """Flat ``window * N + token`` slot feeding each output token ``(c, h, w)``.

    Restates triton_swin3d_layout.py:283-305: undo the shift (``(c - ss) mod C``), add the
    front pad, split into window and in-window coordinates.
    """
    C, H, W = g.C, g.H, g.W
    Wc, Wh, Ww = g.ws
    C1, H1, W1 = g.grid
    c, h, w = np.meshgrid(np.arange(C), np.arange(H), np.arange(W), indexing="ij")
    pc = np.mod(c - g.ss[0], C) + g.pad_front[0]
    ph = np.mod(h - g.ss[1], H) + g.pad_front[1]
    pw = np.mod(w - g.ss[2], W) + g.pad_front[2]
    win = (pc // Wc) * (H1 * W1) + (ph // Wh) * W1 + (pw // Ww)
    tok = (pc % Wc) * (Wh * Ww) + (ph % Wh) * Ww + (pw % Ww)
    return (win * g.window_tokens + tok).reshape(-1).astype(np.int64)


def roll_pad_partition(x: np.ndarray, res, window_size, shift_size) -> np.ndarray:
    """``(B, C, H, W, D)`` -> ``(B * nW, N, D)`` (triton_swin3d_layout.py:58-121)."""
    B, C, H, W, D = x.shape
    g = geometry(res, window_size, shift_size)
    src = partition_source_index(g)
    flat = x.reshape(B, C * H * W, D)
    out = np.zeros((B, g.num_windows, g.window_tokens, D), dtype=x.dtype)
    valid = src >= 0
    out[:, valid, :] = flat[:, src[valid], :]
    return out.reshape(B * g.num_windows, g.window_tokens, D)


def crop_roll_unmerge(windows: np.ndarray, res, window_size, shift_size) -> np.ndarray:
    """``(B * nW, N, D)`` -> ``(B, C, H, W, D)`` (triton_swin3d_layout.py:124-189)."""
    g = geometry(res, window_size, shift_size)
    BnW, N, D = windows.shape
    assert BnW % g.num_windows == 0 and N == g.window_tokens
    B = BnW // g.num_windows
    src = unmerge_source_index(g)
    flat = windows.reshape(B, g.num_windows * N, D)
    return flat[:, src, :].reshape(B, g.C, g.H, g.W, D)


def _merge_groups_3d():
    """swin3d.py:502-514: left/right groups merged per C slice (offset 9 per slice)."""
    pairs = []
    for i_c in range(3):
        for a, b in ((1, 2), (4, 5), (7, 8)):
            pairs.append((a + 9 * i_c, b + 9 * i_c))
    return pairs


def image_group_ids(C, H, W, ws, ss, warped: bool = True) -> np.ndarray:
    """Per-token region id on the padded grid (swin3d.py:566-593).

    ``ws``/``ss`` are the already-adjusted window and shift. Uses the same Python slice objects
    as upstream so that the degenerate cases (a zero shift on one axis) match exactly.
    """
    img = np.zeros((C, H, W), dtype=np.int64)
    cs_ = (slice(0, -ws[0]), slice(-ws[0], -ss[0]), slice(-ss[0], None))
    hs_ = (slice(0, -ws[1]), slice(-ws[1], -ss[1]), slice(-ss[1], None))
    ws_ = (slice(0, -ws[2]), slice(-ws[2], -ss[2]), slice(-ss[2], None))
    cnt = 0
    for c, h, w in itertools.product(cs_, hs_, ws_):
        img[c, h, w] = cnt
        cnt += 1
    if warped:
        for a, b in _merge_groups_3d():
            img[img == a] = b
    pads = ((ws[0] - C % ws[0]) % ws[0], (ws[1] - H % ws[1]) % ws[1], (ws[2] - W % ws[2]) % ws[2])
    (cf, cb), (ht, hb), (wl, wr) = (_split(p) for p in pads)
    return np.pad(img, ((cf, cb), (ht, hb), (wl, wr)), constant_values=cnt)


def window_group_ids(res, window_size, shift_size, warped: bool = True) -> np.ndarray:
    """``(nW, N)`` uint8 region id of each window token; ``None``-equivalent when unshifted.

    Two tokens of a window may attend to each other iff their ids are equal; this is the
    ``attn_mask != 0`` structure of swin3d.py:594-597 in compact form.
    """
    g = geometry(res, window_size, shift_size)
    img = image_group_ids(g.C, g.H, g.W, g.ws, g.ss, warped)
    Cp, Hp, Wp = img.shape
    Wc, Wh, Ww = g.ws
    v = img.reshape(Cp // Wc, Wc, Hp // Wh, Wh, Wp // Ww, Ww)
    v = v.transpose(0, 2, 4, 1, 3, 5).reshape(-1, Wc * Wh * Ww)
    return v.astype(np.uint8)


def shifted_window_mask(res, window_size, shift_size, warped: bool = True) -> np.ndarray:
    """``(nW, N, N)`` float32 additive mask: -100 where the region ids differ, else 0."""
    gid = window_group_ids(res, window_size, shift_size, warped).astype(np.int64)
    diff = gid[:, None, :] - gid[:, :, None]
    return np.where(diff != 0, MASKED_BIAS, 0.0).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# Latitude bands
# ---------------------------------------------------------------------------------------------


def band_split(field_res, window_size, world: int):
    """Token-row ranges of ``world`` bands of whole window rows (first bands get the smaller share)."""
    C, H, W = field_res
    ws, _ = maybe_adjust_windows(tuple(window_size), (0, 0, 0), tuple(field_res))
    rows = H // ws[1]
    assert H % ws[1] == 0 and 1 <= world <= rows
    cuts = [(r * rows) // world for r in range(world + 1)]
    return [(cuts[r] * ws[1], cuts[r + 1] * ws[1]) for r in range(world)]


def _band_shifts(field_res, window_size, shift_size):
    ws, ss = maybe_adjust_windows(tuple(window_size), tuple(shift_size), tuple(field_res))
    return ws, ss


def band_windows_of_field(windows_field: np.ndarray, field_res, window_size, shift_size, h_begin, h_end):
    """Rows ``[h_begin, h_end)`` (token rows) of the field's window grid: ``(B*nW_band, N, D)``."""
    g = geometry(field_res, window_size, shift_size)
    C1, H1, W1 = g.grid
    BnW, N, D = windows_field.shape
    B = BnW // g.num_windows
    v = windows_field.reshape(B, C1, H1, W1, N, D)[:, :, h_begin // g.ws[1]:h_end // g.ws[1]]
    return np.ascontiguousarray(v).reshape(-1, N, D)


def band_partition(x_band: np.ndarray, halo, field_res, window_size, shift_size) -> np.ndarray:
    """Windows of one band: rows ``s..`` of the band followed by the ``s`` halo rows (the next
    band's first rows) form the band's shifted rows; C and W are shifted as in the field."""
    ws, ss = _band_shifts(field_res, window_size, shift_size)
    B, C, Hb, W, D = x_band.shape
    s = ss[1]
    ext = np.concatenate([x_band[:, :, s:], halo], axis=2) if s else x_band
    return roll_pad_partition(ext, (C, Hb, W), ws, (ss[0], 0, ss[2]))


def band_halo_extract(windows_band: np.ndarray, band_res, field_res, window_size, shift_size) -> np.ndarray:
    """The band's last ``s`` shifted rows, un-rolled in C and W: ``(B, C, s, W, D)``."""
    ws, ss = _band_shifts(field_res, window_size, shift_size)
    ext = crop_roll_unmerge(windows_band, tuple(band_res), ws, (ss[0], 0, ss[2]))
    return ext[:, :, band_res[1] - ss[1]:]


def band_unmerge(windows_band: np.ndarray, halo_in, band_res, field_res, window_size, shift_size) -> np.ndarray:
    """Inverse of :func:`band_partition`: ``(B, C, H_band, W, D)``; rows ``0..s-1`` come from
    ``halo_in`` (the previous band's :func:`band_halo_extract`)."""
    ws, ss = _band_shifts(field_res, window_size, shift_size)
    s = ss[1]
    ext = crop_roll_unmerge(windows_band, tuple(band_res), ws, (ss[0], 0, ss[2]))
    if not s:
        return ext
    return np.concatenate([halo_in, ext[:, :, :band_res[1] - s]], axis=2)
