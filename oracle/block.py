"""torch-CPU FP32 restatement of the Swin3D backbone block hot path (test oracle).

Parameters are plain dicts keyed exactly like the upstream ``state_dict`` (for example
``"attn.qkv.weight"``, ``"norm1.ln_modulation.1.bias"``), so a state dict of the upstream
modules, or of the product modules in ``flash_aurora_b200.swin3d``, feeds this oracle directly.

``bf16_mixed=True`` rounds where the upstream ``bf16_mixed`` tier rounds on its GPU path: bfloat16
around the attention and MLP linears (autocast, custom_op_paths.py:188-263, swin3d.py:291-407,
swin3d.py:73-109), bfloat16 probabilities in the window attention's P.V product
(ops/cute/_kernel_bf16.py:418-424), and TF32 operands in the other FP32 linears (time embedding,
AdaLN modulation, patch merge/split: ``_hybrid_linear``); everything else stays FP32. That is
the emulated upstream tier: its drift from the FP32 oracle is the reference's own tier drift, and
it is a tight reference for the BF16 GPU path. With ``bf16_mixed=False`` every step is strict
FP32, the reference for the FP32/3xTF32 tier.

Upstream semantics restated (paths relative to the Flash-Aurora project):

* AdaLN / FiLM                 flash_aurora/aurora/model/film.py:38-48,72-139
* window attention             flash_aurora/aurora/model/swin3d.py:253-409 (SDPA semantics,
                               mask repeated per batch :376-384)
* MLP                          flash_aurora/aurora/model/swin3d.py:40-109 (exact erf GELU)
* Swin3D block                 flash_aurora/aurora/model/swin3d.py:706-815
* PatchMerging3D / Splitting   flash_aurora/aurora/model/swin3d.py:818-919
* backbone forward             flash_aurora/aurora/model/swin3d.py:1231-1313
* lead-time Fourier expansion  flash_aurora/aurora/model/fourier.py:21-131
"""

from __future__ import annotations

import math
from datetime import timedelta

import numpy as np
import torch
import torch.nn.functional as F

from . import layout as L


def _tf32(t: torch.Tensor, on: bool) -> torch.Tensor:
    """Round FP32 to TF32 (10 mantissa bits, to nearest, ties away from zero), when ``on``: the
    operand rounding of a TF32 tensor-core GEMM."""
    if not on:
        return t
    i = t.float().contiguous().view(torch.int32)
    return ((i + 0x1000) & ~0x1FFF).view(torch.float32)


def tf32_linear(x, w, b=None, *, tf32: bool = False):
    """``F.linear`` with TF32 operands (FP32 accumulation) when ``tf32``: upstream's bf16_mixed
    tier runs every FP32 backbone linear outside attention and the MLP (time embedding, AdaLN
    modulation, patch merge/split) as a TF32 GEMM (custom_op_paths.py:188-263, ``_hybrid_linear``)."""
    return F.linear(_tf32(x, tf32), _tf32(w, tf32), b)


def _bf(t: torch.Tensor, on: bool) -> torch.Tensor:
    """Round to bfloat16 and back (round-to-nearest-even), when ``on``."""
    return t.to(torch.bfloat16).to(torch.float32) if on else t


def linear(x, w, b=None, *, bf16: bool = False):
    """``F.linear``; with ``bf16`` the operands and the result are rounded to bfloat16.

    Upstream bf16 autocast (custom_op_paths.py:223-232) casts input and weight to bfloat16,
    accumulates in FP32 and returns bfloat16.
    """
    y = F.linear(_bf(x, bf16), _bf(w, bf16), None if b is None else _bf(b, bf16))
    return _bf(y, bf16)


def adaln_modulation(c, p, prefix, *, tf32: bool = False):
    """film.py:82,117: ``shift, scale = Linear(SiLU(c)).unsqueeze(1).chunk(2)`` (shift first)."""
    mod = tf32_linear(F.silu(c), p[prefix + "ln_modulation.1.weight"], p[prefix + "ln_modulation.1.bias"], tf32=tf32)
    shift, scale = mod.unsqueeze(1).chunk(2, dim=-1)
    return shift, scale


def adaln(x, shift, scale, scale_bias: float = 0.0, eps: float = 1e-5):
    """film.py:97-99: ``LN(x) * (scale_bias + scale) + shift``, LN without affine."""
    return F.layer_norm(x, (x.shape[-1],), eps=eps) * (scale_bias + scale) + shift


def window_attention_core(q, k, v, mask=None, scale=None):
    """``softmax(q k^T * scale + mask[bwin % nW]) v`` for ``(Bwin, H, N, Dh)`` inputs.

    ``mask`` is the ``(nW, N, N)`` additive float mask (swin3d.py:376-384 repeats it per batch,
    window index ``bwin % nW``).
    """
    Bwin, H, N, Dh = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    s = torch.einsum("bhnd,bhmd->bhnm", q, k) * scale
    if mask is not None:
        nW = mask.shape[0]
        idx = torch.arange(Bwin) % nW
        s = s + mask[idx].unsqueeze(1)
    return torch.einsum("bhnm,bhmd->bhnd", torch.softmax(s, dim=-1), v)


def window_attention_core_bf16p(q, k, v, mask=None, scale=None):
    """The upstream bf16 window-attention kernel's rounding (ops/cute/_kernel_bf16.py:418-424,
    501-503): the unnormalised probabilities ``exp(s - rowmax)`` are rounded to bfloat16 before the
    P.V product, which accumulates in FP32; the row sum and the final division stay FP32."""
    Bwin, H, N, Dh = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    s = torch.einsum("bhnd,bhmd->bhnm", q, k) * scale
    if mask is not None:
        idx = torch.arange(Bwin) % mask.shape[0]
        s = s + mask[idx].unsqueeze(1)
    pr = torch.exp(s - s.amax(dim=-1, keepdim=True))
    return torch.einsum("bhnm,bhmd->bhnd", _bf(pr, True), v) / pr.sum(dim=-1, keepdim=True)


def window_attention(xw, mask, p, prefix, num_heads, *, bf16: bool = False, chunk: int = 256):
    """swin3d.py:253-409 for one block: qkv -> attention -> proj (FP32 result). With ``bf16`` the
    attention follows the upstream bf16 kernel's rounding (:func:`window_attention_core_bf16p`).
    Windows are processed ``chunk`` at a time to bound the memory of the logits."""
    Bwin, N, D = xw.shape
    Dh = D // num_heads
    qkv = linear(xw, p[prefix + "qkv.weight"], p[prefix + "qkv.bias"], bf16=bf16)
    qkv = qkv.view(Bwin, N, 3, num_heads, Dh).permute(2, 0, 3, 1, 4)
    core = window_attention_core_bf16p if bf16 else window_attention_core
    if mask is None or mask.shape[0] == Bwin:
        o = torch.cat([core(qkv[0][i:i + chunk], qkv[1][i:i + chunk], qkv[2][i:i + chunk],
                            None if mask is None else mask[i:i + chunk]) for i in range(0, Bwin, chunk)])
    else:
        o = core(qkv[0], qkv[1], qkv[2], mask)
    o = _bf(o, bf16).permute(0, 2, 1, 3).reshape(Bwin, N, D)
    return linear(o, p[prefix + "proj.weight"], p[prefix + "proj.bias"], bf16=bf16)


def mlp(x, p, prefix, *, bf16: bool = False):
    """swin3d.py:73-109: fc1 -> exact GELU -> fc2 (bf16 GELU output under autocast)."""
    h = linear(x, p[prefix + "fc1.weight"], p[prefix + "fc1.bias"], bf16=bf16)
    h = _bf(F.gelu(h), bf16)
    return linear(h, p[prefix + "fc2.weight"], p[prefix + "fc2.bias"], bf16=bf16)


def block_forward(x, c, res, p, *, num_heads, window_size, shift_size, prefix="",
                  bf16_mixed: bool = False, warped: bool = True, eps: float = 1e-5):
    """swin3d.py:706-815 (post-norm Swin3D block) on CPU in FP32.

    ``x`` is ``(B, C*H*W, D)``, ``c`` is ``(B, ctx)``.
    """
    C, H, W = res
    B, Ltok, D = x.shape
    assert Ltok == C * H * W
    g = L.geometry(res, window_size, shift_size)
    mask = None
    if any(s != 0 for s in g.ss):
        mask = torch.from_numpy(L.shifted_window_mask(res, window_size, shift_size, warped))
    xw = torch.from_numpy(L.roll_pad_partition(x.view(B, C, H, W, D).numpy(), res, window_size, shift_size))
    aw = window_attention(xw, mask, p, prefix + "attn.", num_heads, bf16=bf16_mixed)
    a = torch.from_numpy(L.crop_roll_unmerge(aw.numpy(), res, window_size, shift_size)).reshape(B, Ltok, D)
    sh1, sc1 = adaln_modulation(c, p, prefix + "norm1.", tf32=bf16_mixed)
    x = x + adaln(a, sh1, sc1, eps=eps)
    h = mlp(x, p, prefix + "mlp.", bf16=bf16_mixed)
    sh2, sc2 = adaln_modulation(c, p, prefix + "norm2.", tf32=bf16_mixed)
    return x + adaln(h, sh2, sc2, eps=eps)


def patch_merge(x, res, p, prefix, *, tf32: bool = False):
    """swin3d.py:830-861: pad H/W to even, gather 2x2 -> 4D, LayerNorm(4D), Linear(4D->2D)."""
    C, H, W = res
    B, _, D = x.shape
    x = x.view(B, C, H, W, D)
    x = F.pad(x, (0, 0, 0, W % 2, 0, H % 2))  # back/bottom/right only: split of a 1-token pad
    nH, nW_ = x.shape[2], x.shape[3]
    x = x.reshape(B, C, nH // 2, 2, nW_ // 2, 2, D).permute(0, 1, 2, 4, 3, 5, 6)
    x = x.reshape(B, C * (nH // 2) * (nW_ // 2), 4 * D)
    x = F.layer_norm(x, (4 * D,), p[prefix + "norm.weight"], p[prefix + "norm.bias"])
    return tf32_linear(x, p[prefix + "reduction.weight"], tf32=tf32)


def patch_split(x, res, crop, p, prefix, *, tf32: bool = False):
    """swin3d.py:879-919: Linear(D->2D), 2x2 -> spatial, crop, LayerNorm(D/2), Linear."""
    C, H, W = res
    B, _, D = x.shape
    x = tf32_linear(x, p[prefix + "lin1.weight"], tf32=tf32)
    D2 = x.shape[-1]
    x = x.view(B, C, H, W, 2, 2, D2 // 4).permute(0, 1, 2, 4, 3, 5, 6)
    x = x.reshape(B, C, 2 * H, 2 * W, D2 // 4)
    cC, cH, cW = crop
    x = x[:, : x.shape[1] - cC, : x.shape[2] - cH, : x.shape[3] - cW, :]
    x = x.reshape(B, -1, D2 // 4)
    x = F.layer_norm(x, (D2 // 4,), p[prefix + "norm.weight"], p[prefix + "norm.bias"])
    return tf32_linear(x, p[prefix + "lin2.weight"], tf32=tf32)


def lead_time_expansion(hours: torch.Tensor, d: int) -> torch.Tensor:
    """fourier.py:21-131 with ``lower=1/60``, ``upper=24*7*3``: sin/cos features in float64."""
    x = hours.double()
    wl = torch.logspace(math.log10(1 / 60), math.log10(24 * 7 * 3), d // 2, base=10, dtype=torch.float64)
    prod = torch.einsum("...i,j->...ij", x, 2 * np.pi / wl)
    return torch.cat((torch.sin(prod), torch.cos(prod)), dim=-1).float()


def encoder_specs(patch_res, num_layers):
    """swin3d.py:1231-1245: per-stage resolution and the H/W padding of each merge."""
    all_res = [tuple(patch_res)]
    padded = []
    for _ in range(1, num_layers):
        C, H, W = all_res[-1]
        ph, pw = H % 2, W % 2
        padded.append((0, ph, pw))
        all_res.append((C, (H + ph) // 2, (W + pw) // 2))
    padded.append((0, 0, 0))
    return all_res, padded


def backbone_forward(x, lead_time: timedelta, patch_res, p, *, embed_dim, encoder_depths,
                     encoder_num_heads, decoder_depths, decoder_num_heads, window_size,
                     bf16_mixed: bool = False, trace: dict | None = None):
    """swin3d.py:1247-1313: time embedding, encoder stages with merges, decoder stages with
    splits, additive skips for the middle stages, concatenation with the first skip at the end.

    ``trace``: when a dict, it receives the stage outputs under the names upstream's
    error-accumulation trace uses (benchmark/bench_backbone_error_accum.py:180-216):
    ``enc{i}_out`` after each encoder stage (and its merge), ``dec0_out``, ``dec{i}_skip_add``
    for the middle decoder stages and ``dec{n-1}_concat`` for the last."""
    ws = tuple(window_size)
    n_enc, n_dec = len(encoder_depths), len(decoder_depths)
    all_res, padded = encoder_specs(patch_res, n_enc)
    hours = lead_time / timedelta(hours=1)
    lt = torch.full((x.shape[0],), hours, dtype=torch.float32)
    e = lead_time_expansion(lt, embed_dim)
    t32 = bf16_mixed
    c = tf32_linear(F.silu(tf32_linear(e, p["time_mlp.0.weight"], p["time_mlp.0.bias"], tf32=t32)),
                    p["time_mlp.2.weight"], p["time_mlp.2.bias"], tf32=t32)

    def run_layer(x, kind, i, depth, heads, res):
        for j in range(depth):
            ss = (0, 0, 0) if j % 2 == 0 else (ws[0] // 2, ws[1] // 2, ws[2] // 2)
            x = block_forward(x, c, res, p, num_heads=heads, window_size=ws, shift_size=ss,
                              prefix=f"{kind}_layers.{i}.blocks.{j}.", bf16_mixed=bf16_mixed)
        return x

    skips = []
    for i in range(n_enc):
        x = run_layer(x, "encoder", i, encoder_depths[i], encoder_num_heads[i], all_res[i])
        skips.append(x)
        if i < n_enc - 1:
            x = patch_merge(x, all_res[i], p, f"encoder_layers.{i}.downsample.", tf32=bf16_mixed)
        if trace is not None:
            trace[f"enc{i}_out"] = x
    for i in range(n_dec):
        index = n_dec - i - 1
        x = run_layer(x, "decoder", i, decoder_depths[i], decoder_num_heads[i], all_res[index])
        if i < n_dec - 1:
            x = patch_split(x, all_res[index], padded[index - 1], p, f"decoder_layers.{i}.upsample.", tf32=bf16_mixed)
        if 0 < i < n_dec - 1:
            x = x + skips[index - 1]
            tag = f"dec{i}_skip_add"
        elif i == n_dec - 1:
            x = torch.cat([x, skips[0]], dim=-1)
            tag = f"dec{i}_concat"
        else:
            tag = f"dec{i}_out"
        if trace is not None:
            trace[tag] = x
    return x


def relative_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """``||a - b|| / ||b||`` in float64."""
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))
