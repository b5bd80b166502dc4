"""Swin3D backbone block and U-net backbone running on the B200 kernels.

Module structure and ``state_dict`` keys are those of upstream
``flash_aurora/aurora/model/swin3d.py`` / ``film.py`` (``attn.qkv``, ``attn.proj``,
``norm1.ln_modulation.1``, ``mlp.fc1``, ``encoder_layers.i.blocks.j``, ``time_mlp.0``, ...), so an
upstream backbone ``state_dict`` loads unchanged. ``forward`` runs on CUDA only; there is no CPU
path (the upstream pure-PyTorch path is the test oracle, not part of this package).

Per block (upstream swin3d.py:706-815, post-norm), precision ``"bf16_mixed"``:

1. ``fa_roll_pad_partition``: fp32 residual -> bf16 windows (shift + pad + partition + cast); inside a
   stage the previous block's norm2 already wrote them (``fa_adaln_film_partition``).
2. QKV linear, bf16 in/out (``fa_linear_bias_act``: tcgen05 GEMM, CTA pair, bias epilogue).
3. ``fa_window_attention_qkvpacked``: bf16 window attention reading the packed QKV, shifted
   blocks masked by region ids, output in the (window, token, channel) layout.
4. proj linear, bf16 (``fa_linear_bias_act``).
5. ``fa_unmerge_adaln_film``: crop/un-roll/merge of the proj output fused into
   ``x1 = x + AdaLN1(.)`` (fp32), plus a bf16 copy of ``x1`` for fc1.
6. ``fa_linear_bias_act``: fc1 + bias + exact GELU in one tcgen05 kernel (bf16 out).
7. fc2 + ``x2 = x1 + AdaLN2(h)`` (+ the next block's partition): at D = 512 one kernel
   (``fa_linear_adaln_film``, the fc2 output never reaches HBM); elsewhere fc2 on the library GEMM
   at K = 8192 and cuBLAS at K = 4096 (whichever measured faster), then ``fa_adaln_film(_partition)``.

Every rounding point equals the upstream ``bf16_mixed`` tier (custom_op_paths.py:188-263): the
windows and ``x1`` are rounded to bf16 exactly where upstream autocast casts them, and the
attention and linears produce bf16. Precision ``"fp32"`` keeps every tensor fp32 with strict
FP32 GEMMs and 3xTF32 attention; ``"tf32"`` is the same with TF32 GEMMs.
"""

from __future__ import annotations

import contextlib
import math
from datetime import timedelta
from typing import Callable, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .adaln import (
    adaptive_layernorm_film_add_residual_forward,
    adaptive_layernorm_film_add_residual_partition,
    unmerge_adaptive_layernorm_film_add_residual,
    unmerge_adaptive_layernorm_film_add_residual_band,
    adaptive_layernorm_film_add_residual_rows,
)
from . import _lib
from . import recorder as _rec
from .activation import gelu_erf
from .linear import linear_adaln_film_add_residual, linear_bias_act
from .sharding import BandContext
from .swin3d_layout import band_halo_extract, roll_pad_partition_windows, roll_pad_partition_windows_band
from .util import maybe_adjust_windows, window_geometry
from .window_attn import shifted_window_group_ids, window_attn_fwd_cute_qkvpacked
from .workspace_pool import InferenceWorkspacePool

__all__ = [
    "PRECISIONS",
    "AdaptiveLayerNorm",
    "MLP",
    "WindowAttention",
    "Swin3DTransformerBlock",
    "PatchMerging3D",
    "PatchSplitting3D",
    "BasicLayer3D",
    "Swin3DTransformerBackbone",
    "lead_time_expansion",
    "init_random_weights_",
]

PRECISIONS = ("bf16_mixed", "tf32", "fp32")
# In bf16_mixed at D = 512 the fc2 -> norm2 (-> next partition) pair runs as one kernel
# (fa_linear_adaln_film, token rows): measured 3-4 % faster than the pair at config-4 stage 1. The
# same kernel also fuses proj -> unmerge -> norm1 (window rows), but that form measured slower than
# the split pair (0.55-0.62 against 0.38-0.46 ms: its AdaLN phase, 8 warps per SM, is latency-bound
# while a K = 512 GEMM has little tensor work to hide it under), so the block keeps the split pair
# there. Both forms equal the split path up to the summation order of the fp32 row statistics.
FUSE_FC2_ADALN = True
FUSE_PROJ_ADALN = False


def _check_precision(p: str) -> str:
    if p not in PRECISIONS:
        raise ValueError(f"precision must be one of {PRECISIONS}, got {p!r}")
    return p


@contextlib.contextmanager
def _matmul_tf32(enabled: bool):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = enabled
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


class _CastCache:
    """bf16 copies of fp32 parameters, refreshed when the parameter version changes."""

    def __init__(self) -> None:
        self._c: dict[int, tuple[int, torch.Tensor]] = {}

    def get(self, p: torch.Tensor) -> torch.Tensor:
        key = id(p)
        hit = self._c.get(key)
        ver = p._version
        if hit is None or hit[0] != ver or hit[1].device != p.device:
            hit = (ver, p.detach().to(torch.bfloat16))
            self._c[key] = hit
        return hit[1]


class AdaptiveLayerNorm(nn.Module):
    """AdaLN with FiLM modulation (upstream film.py:17-139); state keys ``ln_modulation.1.*``."""

    def __init__(self, dim: int, context_dim: int, scale_bias: float = 0.0) -> None:
        super().__init__()
        self.ln = nn.LayerNorm(dim, elementwise_affine=False)
        self.ln_modulation = nn.Sequential(nn.SiLU(), nn.Linear(context_dim, dim * 2))
        self.scale_bias = scale_bias
        self.init_weights()

    def init_weights(self) -> None:
        nn.init.zeros_(self.ln_modulation[-1].weight)
        nn.init.zeros_(self.ln_modulation[-1].bias)

    def modulation(self, c: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``shift, scale`` of shape ``(B, 1, D)`` in fp32 (film.py:82,117: shift first)."""
        with _matmul_tf32(False):
            mod = F.linear(F.silu(c.float()), self.ln_modulation[1].weight, self.ln_modulation[1].bias)
        shift, scale = mod.unsqueeze(1).chunk(2, dim=-1)
        return shift.contiguous(), scale.contiguous()

    def forward_add_residual(self, residual, x, c, *, out_bf16=None):
        shift, scale = self.modulation(c)
        return adaptive_layernorm_film_add_residual_forward(
            residual, x, scale, shift, float(self.scale_bias), float(self.ln.eps), output_fp32=True,
            out_bf16=out_bf16)


class MLP(nn.Module):
    """fc1 -> exact GELU -> fc2 (upstream swin3d.py:40-109)."""

    def __init__(self, in_features: int, hidden_features: Optional[int] = None,
                 out_features: Optional[int] = None) -> None:
        super().__init__()
        hidden_features = hidden_features or in_features
        out_features = out_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(hidden_features, out_features)


class WindowAttention(nn.Module):
    """W-MSA / SW-MSA parameters (upstream swin3d.py:112-409): ``qkv`` and ``proj`` linears."""

    def __init__(self, dim: int, window_size, num_heads: int, qkv_bias: bool = True) -> None:
        super().__init__()
        assert dim % num_heads == 0, f"dim ({dim}) should be divisible by num_heads ({num_heads})."
        self.dim = dim
        self.window_size = tuple(window_size)
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)


class Swin3DTransformerBlock(nn.Module):
    """Post-norm Swin3D block (upstream swin3d.py:602-815) on the fused B200 path."""

    def __init__(self, dim: int, num_heads: int, time_dim: int, window_size=(2, 7, 7),
                 shift_size=(0, 0, 0), mlp_ratio: float = 4.0, qkv_bias: bool = True,
                 scale_bias: float = 0.0, precision: str = "bf16_mixed") -> None:
        super().__init__()
        self.dim = dim
        self.window_size = tuple(window_size)
        self.shift_size = tuple(shift_size)
        self.num_heads = num_heads
        self.mlp_ratio = mlp_ratio
        self.precision = _check_precision(precision)
        self.norm1 = AdaptiveLayerNorm(dim, time_dim, scale_bias=scale_bias)
        self.attn = WindowAttention(dim, self.window_size, num_heads, qkv_bias=qkv_bias)
        self.norm2 = AdaptiveLayerNorm(dim, time_dim, scale_bias=scale_bias)
        self.mlp = MLP(dim, int(dim * mlp_ratio))
        self._bf16 = _CastCache()

    @staticmethod
    def _linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], bf16: bool) -> torch.Tensor:
        """The block's bf16 linears on this library's tcgen05 GEMM where its tile shape fits (out
        features a multiple of 256, in features a multiple of 64, a bias), else cuBLAS; FP32 tiers
        always use cuBLAS (strict FP32 or TF32)."""
        if bf16 and b is not None and w.shape[0] % 256 == 0 and w.shape[1] % 64 == 0:
            return linear_bias_act(x, w, b, act="none")
        return F.linear(x, w, b)

    def _w(self, lin: nn.Linear, bf16: bool):
        if not bf16:
            return lin.weight, lin.bias
        return self._bf16.get(lin.weight), (self._bf16.get(lin.bias) if lin.bias is not None else None)

    def forward(self, x: torch.Tensor, c: torch.Tensor, res, rollout_step: int = 0,
                warped: bool = True, band: Optional[BandContext] = None,
                windows: Optional[torch.Tensor] = None,
                next_windows: Optional[tuple] = None,
                mods: Optional[tuple] = None,
                halo_prefetch: Optional[int] = None) -> torch.Tensor:
        """``x (B, C*H*W, D)`` fp32, ``c (B, ctx)`` -> ``(B, C*H*W, D)`` fp32.

        With ``band`` (a :class:`~flash_aurora_b200.sharding.BandContext`), ``x`` and ``res`` are
        this rank's latitude band of the field ``band.field_res``: the window geometry and mask are
        the field's, a shifted block exchanges its half-window halo rows with the neighbouring
        bands, and the result equals the band's rows of the unsharded block.

        ``mods``: ``(shift1, scale1, shift2, scale2)`` of the two norms, computed for all blocks at
        once by the backbone (otherwise each norm computes its own).

        ``windows``: this block's partition of ``x``, already written by the previous block's
        norm2 (the partition is then skipped). ``next_windows = (shift_size, buffer)``: also write
        the output into ``buffer`` in the window layout of a following block with that shift
        (same window size); ``buffer`` keeps zeros in its pad slots.

        ``halo_prefetch = s`` (with ``band``): the next block is shifted by ``s`` rows. Its forward
        halo (the first ``s`` rows of this block's output) is normalised first and handed to the
        band's side stream while the other rows are normalised.
        """
        if not x.is_cuda:
            raise RuntimeError("Swin3DTransformerBlock.forward requires CUDA tensors (no CPU path).")
        C, H, W = res
        B, L, D = x.shape
        assert L == C * H * W, f"Wrong feature size: {L} vs {C}x{H}x{W}={C * H * W}"
        if x.dtype != torch.float32:
            x = x.float()
        x = x.contiguous()
        if band is not None and tuple(res) != band.res:
            raise ValueError(f"res {tuple(res)} is not the band's resolution {band.res}")
        if halo_prefetch and (band is None or not 0 < halo_prefetch < H):
            raise ValueError("halo_prefetch needs a band taller than the halo")
        field_res = band.field_res if band is not None else tuple(res)
        ws, ss = maybe_adjust_windows(self.window_size, self.shift_size, field_res)
        if band is not None:
            gids = band.group_ids(self.window_size, self.shift_size, warped, x.device)
        elif any(s != 0 for s in ss):
            gids = shifted_window_group_ids(tuple(res), self.window_size, self.shift_size, warped, x.device)
        else:
            gids = None
        bf16 = self.precision == "bf16_mixed"
        act = torch.bfloat16 if bf16 else torch.float32
        heads = self.num_heads
        if mods is not None:
            sh1, sc1, sh2, sc2 = mods
        else:
            sh1, sc1 = self.norm1.modulation(c)
            sh2, sc2 = self.norm2.modulation(c)
        eps = float(self.norm1.ln.eps)
        # Algorithmic sizes of this call, for the optional step recorder (recorder.py): L tokens,
        # T window slots (pads included), activation element size e.
        e = 2 if bf16 else 4
        with _matmul_tf32(self.precision == "tf32"):
            x5 = x.view(B, C, H, W, D)
            if windows is not None:
                if band is not None:
                    raise ValueError("prepartitioned windows are not used with latitude bands")
                xw = windows
            elif band is None:
                ev = _rec.begin()
                xw = roll_pad_partition_windows(x5, res, self.window_size, self.shift_size, out_dtype=act)
                _rec.end("partition", ev, L * D * 4 * B + xw.numel() * e)
            else:
                # The halo rows travel already rounded to the windows' dtype (bf16 in bf16_mixed:
                # half the bytes, bit-identical windows since the rounding commutes with the gather).
                halo = band.halo_forward(x5, ss[1], dtype=act) if ss[1] else None
                xw = roll_pad_partition_windows_band(x5, halo, field_res, self.window_size, self.shift_size,
                                                     out_dtype=act)
            T = xw.shape[0] * xw.shape[1]
            wq, bq = self._w(self.attn.qkv, bf16)
            ev = _rec.begin()
            qkv = self._linear(xw, wq, bq, bf16)
            _rec.end("qkv_gemm", ev, (T * D + 3 * D * D + 3 * T * D) * e, 2 * T * D * 3 * D)
            ev = _rec.begin()
            a = window_attn_fwd_cute_qkvpacked(qkv, heads, group_ids=gids, output_layout="bnc")
            Nw = xw.shape[1]
            _rec.end("attention", ev, 4 * T * D * e, 4 * xw.shape[0] * heads * Nw * Nw * (D // heads))
            wp, bp = self._w(self.attn.proj, bf16)
            x1_bf16 = torch.empty(B, L, D, device=x.device, dtype=torch.bfloat16) if bf16 else None
            fusable = bf16 and band is None and D == 512
            fuse = FUSE_PROJ_ADALN and fusable and bp is not None
            if fuse:
                # proj + crop/un-roll/merge + norm1 + residual in one kernel (the proj output stays
                # on chip); also writes the bf16 copy of x1 for fc1.
                ev = _rec.begin()
                x1 = linear_adaln_film_add_residual(
                    a, wp, bp, x, sc1, sh1, res, self.window_size, self.shift_size, rows="windows",
                    scale_bias=float(self.norm1.scale_bias), eps=eps, out_bf16=x1_bf16)
                _rec.end("proj_adaln1", ev, (T * D + D * D) * e + B * L * D * (4 + 4 + 2), 2 * T * D * D)
            else:
                ev = _rec.begin()
                a = self._linear(a, wp, bp, bf16)
                _rec.end("proj_gemm", ev, (2 * T * D + D * D) * e, 2 * T * D * D)
            ev = _rec.begin()
            if fuse:
                pass
            elif band is None:
                x1 = unmerge_adaptive_layernorm_film_add_residual(
                    a, x, sc1, sh1, res, self.window_size, self.shift_size, float(self.norm1.scale_bias), eps,
                    out_bf16=x1_bf16)
            elif not ss[1] or not band.overlap:
                halo_in = None
                if ss[1]:
                    rows = band_halo_extract(a, res, field_res, self.window_size, self.shift_size,
                                             out=band.buffer("back_send", (B, C, ss[1], W, D), a.dtype, a.device))
                    halo_in = band.halo_back(rows)
                x1 = unmerge_adaptive_layernorm_film_add_residual_band(
                    a, halo_in, x, sc1, sh1, res, field_res, self.window_size, self.shift_size,
                    float(self.norm1.scale_bias), eps, out_bf16=x1_bf16)
            else:
                # The band's last s shifted rows go to the next band while the rows that need no
                # halo are normalised; the first s rows wait for the previous band's rows.
                s1 = ss[1]
                rows = band_halo_extract(a, res, field_res, self.window_size, self.shift_size,
                                         out=band.buffer("back_send", (B, C, s1, W, D), a.dtype, a.device))
                pending = band.halo_back_async(rows)
                x1 = torch.empty(B, L, D, device=x.device, dtype=torch.float32)
                nargs = (res, field_res, self.window_size, self.shift_size, float(self.norm1.scale_bias), eps)
                unmerge_adaptive_layernorm_film_add_residual_band(
                    a, None, x, sc1, sh1, *nargs, out_bf16=x1_bf16, out=x1, rows=(s1, H - s1))
                unmerge_adaptive_layernorm_film_add_residual_band(
                    a, pending.wait(), x, sc1, sh1, *nargs, out_bf16=x1_bf16, out=x1, rows=(0, s1))
            if not fuse:
                # windows (non-pad tokens) + fp32 residual read, fp32 output (+ bf16 copy) written
                _rec.end("adaln1_unmerge", ev, B * L * D * (e + 4 + 4 + (2 if bf16 else 0)))
            w1, b1 = self._w(self.mlp.fc1, bf16)
            hid = w1.shape[0]
            ev = _rec.begin()
            if bf16 and b1 is not None and w1.shape[0] % 256 == 0 and w1.shape[1] % 64 == 0:
                # fc1 + bias + GELU in one tensor-core kernel (GELU on the fp32 sum).
                h = linear_bias_act(x1_bf16, w1, b1, act="gelu")
            else:
                h = F.linear(x1_bf16 if bf16 else x1, w1, b1)
                h = gelu_erf(h, inplace=True)
            _rec.end("fc1_gelu_gemm", ev, (B * L * D + hid * D + B * L * hid) * e, 2 * B * L * D * hid)
            w2, b2 = self._w(self.mlp.fc2, bf16)
            if FUSE_FC2_ADALN and fusable and b2 is not None and w2.shape[1] % 32 == 0:
                # fc2 + norm2 + residual (+ the next block's partition) in one kernel.
                ev = _rec.begin()
                nxt = None
                if next_windows is not None:
                    nxt = next_windows
                y = linear_adaln_film_add_residual(
                    h, w2, b2, x1, sc2, sh2, res, self.window_size, self.shift_size, rows="tokens",
                    scale_bias=float(self.norm2.scale_bias), eps=eps, next_windows=nxt)
                _rec.end("fc2_adaln2", ev, (B * L * hid + hid * D) * e + B * L * D * (4 + 4 + (2 if nxt else 0)),
                         2 * B * L * D * hid)
                return y
            ev = _rec.begin()
            if bf16 and b2 is not None and w2.shape[0] % 256 == 0 and w2.shape[1] >= 8192:
                # Measured per stage: the library GEMM wins at K = 8192 (stage 3), cuBLAS at K = 4096.
                h = linear_bias_act(h, w2, b2, act="none")
            else:
                h = F.linear(h, w2, b2)
            _rec.end("fc2_gemm", ev, (B * L * hid + hid * D + B * L * D) * e, 2 * B * L * D * hid)
            ev = _rec.begin()
            if next_windows is not None:
                if band is not None:
                    raise ValueError("next-block windows are not produced with latitude bands")
                next_shift, buf = next_windows
                y = adaptive_layernorm_film_add_residual_partition(
                    x1, h, sc2, sh2, res, self.window_size, next_shift, buf, float(self.norm2.scale_bias), eps)
                _rec.end("adaln2_partition", ev, B * L * D * (e + 4 + 4 + e))
                return y
            if halo_prefetch:
                # The next shifted block's forward halo first, then the rest of the rows while it
                # travels.
                y = torch.empty(B, L, D, device=x.device, dtype=torch.float32)
                sb2 = float(self.norm2.scale_bias)
                adaptive_layernorm_film_add_residual_rows(x1, h, sc2, sh2, res, (0, halo_prefetch), sb2, eps, out=y)
                band.prefetch_forward_halo(y.view(B, C, H, W, D), halo_prefetch, dtype=act)
                adaptive_layernorm_film_add_residual_rows(x1, h, sc2, sh2, res, (halo_prefetch, H - halo_prefetch),
                                                          sb2, eps, out=y)
            else:
                y = adaptive_layernorm_film_add_residual_forward(
                    x1, h, sc2, sh2, float(self.norm2.scale_bias), eps, output_fp32=True)
            _rec.end("adaln2", ev, B * L * D * (e + 4 + 4))
            return y


class PatchMerging3D(nn.Module):
    """2x2 patch merge + LayerNorm(4D) + Linear(4D -> 2D) (upstream swin3d.py:818-861)."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.dim = dim
        self.reduction = nn.Linear(4 * dim, 2 * dim, bias=False)
        self.norm = nn.LayerNorm(4 * dim)

    def forward(self, x: torch.Tensor, input_resolution) -> torch.Tensor:
        C, H, W = input_resolution
        B, L, D = x.shape
        assert L == C * H * W and H > 1 and W > 1
        if x.dtype == torch.float32 and D % 8 == 0 and 4 * D <= 4096:
            # pad + 2x2 gather + LayerNorm(4D) in one kernel (fa_patch_merge_ln)
            x = x.contiguous()
            out = torch.empty(B, C * ((H + 1) // 2) * ((W + 1) // 2), 4 * D, device=x.device, dtype=torch.float32)
            rc = _lib.load().fa_patch_merge_ln(
                x.data_ptr(), out.data_ptr(), self.norm.weight.float().contiguous().data_ptr(),
                self.norm.bias.float().contiguous().data_ptr(), B, C, H, W, D, float(self.norm.eps),
                _lib.stream_ptr(x.device))
            _lib.check(rc, "PatchMerging3D")
            return self.reduction(out)
        x = x.view(B, C, H, W, D)
        x = F.pad(x, (0, 0, 0, W % 2, 0, H % 2))  # swin3d.py:839: a 1-token pad goes to the back
        nH, nW = x.shape[2], x.shape[3]
        x = x.reshape(B, C, nH // 2, 2, nW // 2, 2, D).permute(0, 1, 2, 4, 3, 5, 6)
        x = x.reshape(B, C * (nH // 2) * (nW // 2), 4 * D)
        return self.reduction(self.norm(x))


class PatchSplitting3D(nn.Module):
    """Linear(D -> 2D) + 2x2 split + crop + LayerNorm(D/2) + Linear (upstream swin3d.py:864-919)."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.dim = dim
        assert dim % 2 == 0, f"dim ({dim}) should be divisible by 2."
        self.lin1 = nn.Linear(dim, dim * 2, bias=False)
        self.lin2 = nn.Linear(dim // 2, dim // 2, bias=False)
        self.norm = nn.LayerNorm(dim // 2)

    def forward(self, x: torch.Tensor, input_resolution, crop=(0, 0, 0)) -> torch.Tensor:
        C, H, W = input_resolution
        x = self.lin1(x)
        B, L, D = x.shape
        assert L == C * H * W and D % 4 == 0
        Dq = D // 4
        if x.dtype == torch.float32 and Dq % 8 == 0 and Dq <= 4096:
            # 2x2 split + crop + LayerNorm(D/4) in one kernel (fa_patch_split_ln)
            cC, cH, cW = (int(v) for v in crop)
            x = x.contiguous()
            out = torch.empty(B, (C - cC) * (2 * H - cH) * (2 * W - cW), Dq, device=x.device, dtype=torch.float32)
            rc = _lib.load().fa_patch_split_ln(
                x.data_ptr(), out.data_ptr(), self.norm.weight.float().contiguous().data_ptr(),
                self.norm.bias.float().contiguous().data_ptr(), B, C, H, W, Dq, _lib.i32x3((cC, cH, cW)),
                float(self.norm.eps), _lib.stream_ptr(x.device))
            _lib.check(rc, "PatchSplitting3D")
            return self.lin2(out)
        x = x.view(B, C, H, W, 2, 2, D // 4).permute(0, 1, 2, 4, 3, 5, 6).reshape(B, C, 2 * H, 2 * W, D // 4)
        cC, cH, cW = crop
        x = x[:, : x.shape[1] - cC, : x.shape[2] - cH, : x.shape[3] - cW, :]
        x = x.reshape(B, -1, D // 4)
        return self.lin2(self.norm(x))


class BasicLayer3D(nn.Module):
    """One stage: ``depth`` blocks alternating unshifted / shifted windows (swin3d.py:922-1068)."""

    def __init__(self, dim: int, depth: int, num_heads: int, ws, time_dim: int, mlp_ratio: float = 4.0,
                 qkv_bias: bool = True, downsample: Optional[type] = None, upsample: Optional[type] = None,
                 scale_bias: float = 0.0, precision: str = "bf16_mixed") -> None:
        super().__init__()
        if downsample is not None and upsample is not None:
            raise ValueError("Cannot set both `downsample` and `upsample`.")
        self.dim = dim
        self.depth = depth
        ws = tuple(ws)
        self.blocks = nn.ModuleList([
            Swin3DTransformerBlock(
                dim=dim, num_heads=num_heads, window_size=ws,
                shift_size=(0, 0, 0) if i % 2 == 0 else (ws[0] // 2, ws[1] // 2, ws[2] // 2),
                time_dim=time_dim, mlp_ratio=mlp_ratio, qkv_bias=qkv_bias, scale_bias=scale_bias,
                precision=precision)
            for i in range(depth)
        ])
        self.downsample = downsample(dim=dim) if downsample is not None else None
        self.upsample = upsample(dim=dim) if upsample is not None else None

    def forward(self, x, c, res, crop=(0, 0, 0), rollout_step: int = 0,
                band: Optional[BandContext] = None, mods: Optional[list] = None):
        """``band``: run the blocks on this rank's latitude band of the stage's field (a stage
        with a patch merge or split is not sharded: those change the band geometry)."""
        if band is not None and (self.downsample is not None or self.upsample is not None):
            raise ValueError("latitude-band sharding covers block stacks without patch merge/split")
        if mods is None:
            mods = [None] * len(self.blocks)
        if band is not None or not x.is_cuda:
            for i, (blk, m) in enumerate(zip(self.blocks, mods)):
                pre = None
                if band is not None and band.overlap and i + 1 < len(self.blocks):
                    # A shifted next block: its forward halo leaves while this block finishes.
                    nb = self.blocks[i + 1]
                    _, nss = maybe_adjust_windows(nb.window_size, nb.shift_size, band.field_res)
                    pre = nss[1] or None
                x = blk(x, c, res, rollout_step, band=band, mods=m, halo_prefetch=pre)
        else:
            # Each block's norm2 also writes the next block's windows (norm2 + partition fused);
            # one zero-filled buffer per stage keeps the pad slots zero.
            windows = None
            for i, blk in enumerate(self.blocks):
                nxt = self.blocks[i + 1] if i + 1 < len(self.blocks) else None
                buf = self._window_buffer(x, res, nxt) if nxt is not None else None
                x = blk(x, c, res, rollout_step, windows=windows,
                        next_windows=(nxt.shift_size, buf) if nxt is not None else None, mods=mods[i])
                windows = buf
        if self.downsample is not None:
            return self.downsample(x, res), x
        if self.upsample is not None:
            return self.upsample(x, res, crop), x
        return x, None

    def _window_buffer(self, x: torch.Tensor, res, blk: "Swin3DTransformerBlock") -> torch.Tensor:
        """Zero-filled ``(B * nW, N, D)`` window buffer for ``blk``'s geometry, kept per shape."""
        B, _, D = x.shape
        act = torch.bfloat16 if blk.precision == "bf16_mixed" else torch.float32
        _, _, _, _, nW, N = window_geometry(tuple(res), blk.window_size, blk.shift_size)
        key = (B, tuple(res), blk.window_size, D, act, str(x.device))
        cache = self.__dict__.setdefault("_win_bufs", {})
        buf = cache.get(key)
        if buf is None:
            buf = torch.zeros(B * nW, N, D, dtype=act, device=x.device)
            cache[key] = buf
        return buf

    def init_respostnorm(self) -> None:
        for blk in self.blocks:
            blk.norm1.init_weights()
            blk.norm2.init_weights()


class Basic3DEncoderLayer(BasicLayer3D):
    """Encoder stage (same as :class:`BasicLayer3D`)."""


class Basic3DDecoderLayer(BasicLayer3D):
    """Decoder stage (same as :class:`BasicLayer3D`)."""


def lead_time_expansion(hours: torch.Tensor, d: int) -> torch.Tensor:
    """Fourier lead-time features (upstream fourier.py, ``FourierExpansion(1/60, 24*7*3)``):
    ``d // 2`` log-spaced wavelengths, ``[sin, cos]`` of ``2 pi x / wavelength`` in float64."""
    if d % 2:
        raise ValueError("The dimensionality must be a multiple of two.")
    x = hours.double()
    wl = torch.logspace(math.log10(1 / 60), math.log10(24 * 7 * 3), d // 2, base=10, device=x.device,
                        dtype=torch.float64)
    prod = torch.einsum("...i,j->...ij", x, 2 * np.pi / wl)
    return torch.cat((torch.sin(prod), torch.cos(prod)), dim=-1).float()


class Swin3DTransformerBackbone(nn.Module):
    """Swin3D U-net backbone (upstream swin3d.py:1079-1313) on the B200 block path."""

    def __init__(self, embed_dim: int = 96, encoder_depths=(2, 2, 6, 2), encoder_num_heads=(3, 6, 12, 24),
                 decoder_depths=(2, 6, 2, 2), decoder_num_heads=(24, 12, 6, 3), window_size=7,
                 mlp_ratio: float = 4.0, qkv_bias: bool = True, precision: str = "bf16_mixed",
                 workspace_pool: Optional[InferenceWorkspacePool] = None) -> None:
        super().__init__()
        self.precision = _check_precision(precision)
        self.workspace_pool = workspace_pool
        # Called with the first encoder layer's output, the skip half of the final concatenation,
        # as soon as it exists (a serving pipeline starts its download there); None: nothing.
        self.skip_hook: Optional[Callable[[torch.Tensor], None]] = None
        self.window_size = tuple(window_size) if isinstance(window_size, (tuple, list)) else (window_size,) * 3
        self.num_encoder_layers = len(encoder_depths)
        self.num_decoder_layers = len(decoder_depths)
        self.embed_dim = embed_dim
        self.mlp_ratio = mlp_ratio
        self.time_mlp = nn.Sequential(nn.Linear(embed_dim, embed_dim), nn.SiLU(), nn.Linear(embed_dim, embed_dim))
        assert sum(encoder_depths) == sum(decoder_depths)
        self.encoder_layers = nn.ModuleList([
            Basic3DEncoderLayer(dim=int(embed_dim * 2 ** i), depth=encoder_depths[i], num_heads=encoder_num_heads[i],
                                ws=self.window_size, time_dim=embed_dim, mlp_ratio=mlp_ratio, qkv_bias=qkv_bias,
                                downsample=PatchMerging3D if i < self.num_encoder_layers - 1 else None,
                                precision=precision)
            for i in range(self.num_encoder_layers)
        ])
        self.decoder_layers = nn.ModuleList()
        for i in range(self.num_decoder_layers):
            e = self.num_decoder_layers - i - 1
            self.decoder_layers.append(Basic3DDecoderLayer(
                dim=int(embed_dim * 2 ** e), depth=decoder_depths[i], num_heads=decoder_num_heads[i],
                ws=self.window_size, time_dim=embed_dim, mlp_ratio=mlp_ratio, qkv_bias=qkv_bias,
                upsample=PatchSplitting3D if i < self.num_decoder_layers - 1 else None, precision=precision))

    def set_precision(self, precision: str) -> None:
        self.precision = _check_precision(precision)
        for m in self.modules():
            if isinstance(m, Swin3DTransformerBlock):
                m.precision = precision

    def get_encoder_specs(self, patch_res):
        """Per-stage resolution and merge padding (upstream swin3d.py:1231-1245)."""
        all_res = [tuple(patch_res)]
        padded = []
        for _ in range(1, self.num_encoder_layers):
            C, H, W = all_res[-1]
            ph, pw = H % 2, W % 2
            padded.append((0, ph, pw))
            all_res.append((C, (H + ph) // 2, (W + pw) // 2))
        padded.append((0, 0, 0))
        return all_res, padded

    def _modulations(self, c: torch.Tensor) -> dict:
        """(shift1, scale1, shift2, scale2) of every block, from one SiLU and one fp32 GEMM over the
        concatenated modulation weights of all norms (film.py:82,117: shift first), instead of
        two tiny GEMVs per block. The concatenation is cached and rebuilt when a weight changes."""
        norms = []
        layers = list(self.encoder_layers) + list(self.decoder_layers)
        for layer in layers:
            for blk in layer.blocks:
                norms.extend((blk.norm1, blk.norm2))
        lins = [n.ln_modulation[1] for n in norms]
        key = tuple((id(l.weight), l.weight._version, id(l.bias), l.bias._version, str(l.weight.device))
                    for l in lins)
        cache = self.__dict__.get("_mod_cat")
        if cache is None or cache[0] != key:
            w = torch.cat([l.weight.detach() for l in lins], dim=0).float().contiguous()
            b = torch.cat([l.bias.detach() for l in lins], dim=0).float().contiguous()
            cache = (key, w, b, [l.weight.shape[0] for l in lins])
            self.__dict__["_mod_cat"] = cache
        _, w, b, sizes = cache
        with _matmul_tf32(False):
            allmod = F.linear(F.silu(c.float()), w, b)
        parts = allmod.unsqueeze(1).split(sizes, dim=-1)
        out: dict = {}
        k = 0
        for layer in layers:
            per_block = []
            for _ in layer.blocks:
                s1, c1 = parts[k].chunk(2, dim=-1)
                s2, c2 = parts[k + 1].chunk(2, dim=-1)
                per_block.append((s1.contiguous(), c1.contiguous(), s2.contiguous(), c2.contiguous()))
                k += 2
            out[layer] = per_block
        return out

    def time_embedding(self, lead_time: timedelta, batch: int, device) -> torch.Tensor:
        hours = lead_time / timedelta(hours=1)
        lt = torch.full((batch,), hours, dtype=torch.float32, device=device)
        with _matmul_tf32(False):
            return self.time_mlp(lead_time_expansion(lt, self.embed_dim))

    def forward(self, x: torch.Tensor, lead_time: timedelta, rollout_step: int, patch_res) -> torch.Tensor:
        assert x.shape[1] == patch_res[0] * patch_res[1] * patch_res[2], "Input shape does not match patch size."
        assert patch_res[0] % self.window_size[0] == 0
        if not x.is_cuda:
            raise RuntimeError("Swin3DTransformerBackbone.forward requires CUDA tensors (no CPU path).")
        all_res, padded = self.get_encoder_specs(patch_res)
        c = self.time_embedding(lead_time, x.shape[0], x.device)
        mods = self._modulations(c)
        # Stage-boundary linears follow the tier: TF32 in bf16_mixed/tf32 (upstream hybrid
        # routing, custom_op_paths.py:234-243), strict FP32 in fp32.
        with _matmul_tf32(self.precision != "fp32"):
            skips = []
            for i, layer in enumerate(self.encoder_layers):
                x, x_unscaled = layer(x, c, all_res[i], rollout_step=rollout_step, mods=mods[layer])
                skips.append(x_unscaled)
                if i == 0 and self.skip_hook is not None:
                    self.skip_hook(x_unscaled)
            for i, layer in enumerate(self.decoder_layers):
                index = self.num_decoder_layers - i - 1
                x, _ = layer(x, c, all_res[index], padded[index - 1], rollout_step=rollout_step,
                             mods=mods[layer])
                if 0 < i < self.num_decoder_layers - 1:
                    x = x + skips[index - 1]
                elif i == self.num_decoder_layers - 1:
                    x = torch.cat([x, skips[0]], dim=-1)
        return x


@torch.no_grad()
def init_random_weights_(module: nn.Module, std: float = 0.02, generator: Optional[torch.Generator] = None) -> None:
    """Random init used by the benchmarks: every Linear weight ~N(0, std), biases 0, LayerNorm
    weight 1 / bias 0. Unlike the upstream init this also draws the AdaLN modulation, which
    upstream zero-initialises (film.py:45-48) and which would make every block an identity."""
    for m in module.modules():
        if isinstance(m, nn.Linear):
            m.weight.normal_(0.0, std, generator=generator)
            if m.bias is not None:
                m.bias.zero_()
        elif isinstance(m, nn.LayerNorm) and m.weight is not None:
            m.weight.fill_(1.0)
            m.bias.zero_()
