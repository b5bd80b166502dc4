"""GPU parity of the window attention kernels against the oracle (FP32 SDPA semantics with the
upstream -100 mask), on the upstream test shapes, real Swin masks and edge cases.

Tolerances: bf16 I/O vs FP32 reference on the same inputs: rtol = atol = 2e-2 (the upstream
test_cute_window_attn.py:308-334 bound); FP32 I/O (3xTF32) vs strict FP32: relative L2 <= 1e-5
and max abs <= 1e-5 (the north-star FP32-tier bound)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import flash_aurora_b200 as fa
from oracle import block as OB
from oracle import layout as OL

pytestmark = pytest.mark.gpu
P = fa.WinAttnPrecision

# Upstream AURORA_SHAPES / EXTRA_SHAPES restricted to N <= 144 (Bwin, H, N, Dh, nW).
SHAPES = [(16, 8, 144, 64, 4), (8, 16, 144, 64, 4), (4, 32, 144, 64, 4), (4, 8, 64, 64, 2), (6, 4, 96, 64, 3)]


def _qkv(Bwin, H, N, Dh, seed=42, scale=0.1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(Bwin, H, N, Dh, generator=g) * scale for _ in range(3)]


def _half_bias(nW, N):
    b = torch.zeros(nW, N, N)
    b[:, N // 2:, : N // 2] = -100.0
    return b


def _rel_l2(a, b):
    return OB.relative_l2(a.cpu().float(), b.cpu().float())


@pytest.mark.parametrize("Bwin,H,N,Dh,nW", SHAPES)
@pytest.mark.parametrize("has_bias", [False, True])
def test_bf16_close_to_fp32(Bwin, H, N, Dh, nW, has_bias):
    q, k, v = _qkv(Bwin, H, N, Dh)
    bias = _half_bias(nW, N) if has_bias else None
    ref = OB.window_attention_core(q, k, v, bias)
    out = fa.window_attn_fwd_cute(q.bfloat16().cuda(), k.bfloat16().cuda(), v.bfloat16().cuda(),
                                  bias.cuda() if bias is not None else None, precision=P.BF16_MIXED)
    assert out.dtype == torch.bfloat16 and out.shape == (Bwin, H, N, Dh)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Bwin,H,N,Dh,nW", SHAPES)
@pytest.mark.parametrize("has_bias", [False, True])
def test_fp32_3xtf32_close_to_strict_fp32(Bwin, H, N, Dh, nW, has_bias):
    q, k, v = _qkv(Bwin, H, N, Dh)
    bias = _half_bias(nW, N) if has_bias else None
    ref = OB.window_attention_core(q.double(), k.double(), v.double(), bias.double() if bias is not None else None)
    out = fa.window_attn_fwd_cute(q.cuda(), k.cuda(), v.cuda(), bias.cuda() if bias is not None else None,
                                  precision=P.TF32_ACC_FP32)
    assert out.dtype == torch.float32
    assert _rel_l2(out, ref) <= 1e-5
    assert (out.cpu().double() - ref).abs().max().item() <= 1e-5


@pytest.mark.parametrize("act_scale", [1.0, 4.0, 5.0])
def test_large_activations_with_swin_mask(act_scale):
    # Upstream test_cute_window_attn.py:206-288 (max-abs bounds at production-scale logits).
    Bwin, H, N, Dh, nW = 6, 8, 144, 64, 3
    q, k, v = _qkv(Bwin, H, N, Dh, scale=act_scale)
    bias = _half_bias(nW, N)
    ref = OB.window_attention_core(q.double(), k.double(), v.double(), bias.double())
    o32 = fa.window_attn_fwd_cute(q.cuda(), k.cuda(), v.cuda(), bias.cuda(), precision=P.TF32_ACC_FP32)
    assert (o32.cpu().double() - ref).abs().max().item() < {1.0: 0.05, 4.0: 0.16, 5.0: 0.26}[act_scale] / 100
    qb, kb, vb = (t.bfloat16() for t in (q, k, v))
    refb = OB.window_attention_core(qb.double(), kb.double(), vb.double(), bias.double())
    ob = fa.window_attn_fwd_cute(qb.cuda(), kb.cuda(), vb.cuda(), bias.cuda(), precision=P.BF16_MIXED)
    assert (ob.cpu().double() - refb).abs().max().item() < {1.0: 0.02, 4.0: 0.8, 5.0: 1.7}[act_scale]


@pytest.mark.parametrize("res", [(4, 36, 72), (4, 45, 90), (3, 13, 25)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_real_swin_mask_groups_equal_bias(res, dtype):
    ws, ss = (2, 6, 12), (1, 3, 6)
    gm = OL.geometry(res, ws, ss)
    nW, N, H = gm.num_windows, gm.window_tokens, 2
    q, k, v = _qkv(2 * nW, H, N, 64, seed=3, scale=1.0)
    bias = torch.from_numpy(OL.shifted_window_mask(res, ws, ss))
    gids = fa.shifted_window_group_ids(res, ws, ss, device="cuda")
    prec = P.BF16_MIXED if dtype == torch.bfloat16 else P.TF32_ACC_FP32
    qc, kc, vc = (t.to(dtype).cuda() for t in (q, k, v))
    a = fa.window_attn_fwd_cute(qc, kc, vc, bias.cuda(), precision=prec)
    b = fa.window_attn_fwd_cute(qc, kc, vc, precision=prec, group_ids=gids)
    ref = OB.window_attention_core(*(t.to(dtype).double() for t in (q, k, v)), bias.double())
    if dtype == torch.float32:
        assert torch.equal(a, b)
        assert _rel_l2(a, ref) <= 1e-5
    else:
        # bf16: the region ids go through the mask UMMA (same-region logits raised by 100/scale),
        # the float bias through a per-logit mask; both are the upstream softmax, rounded apart.
        assert _rel_l2(a, ref) <= 1e-2 and _rel_l2(b, ref) <= 1e-2
        assert (a.float() - b.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("has_bias", [False, True])
def test_qkvpacked_matches_regular(dtype, has_bias):
    # Upstream test_cute_window_attn.py:359-464: packed == regular, bit-exact, both layouts.
    Bwin, H, N, Dh, nW = 6, 8, 144, 64, 3
    q, k, v = (t.to(dtype).cuda() for t in _qkv(Bwin, H, N, Dh, scale=1.0))
    bias = _half_bias(nW, N).cuda() if has_bias else None
    qkv = torch.empty(Bwin, N, 3 * H * Dh, device="cuda", dtype=dtype)
    view = qkv.view(Bwin, N, 3, H, Dh)
    for i, t in enumerate((q, k, v)):
        view[:, :, i].copy_(t.permute(0, 2, 1, 3))
    prec = P.BF16_MIXED if dtype == torch.bfloat16 else P.TF32_ACC_FP32
    regular = fa.window_attn_fwd_cute(q, k, v, bias, precision=prec)
    packed = fa.window_attn_fwd_cute_qkvpacked(qkv, H, bias=bias)
    assert torch.equal(packed, regular)
    bnc = fa.window_attn_fwd_cute_qkvpacked(qkv, H, bias=bias, output_layout="bnc")
    assert bnc.shape == (Bwin, N, H * Dh) and bnc.is_contiguous()
    assert torch.equal(bnc, regular.permute(0, 2, 1, 3).reshape(Bwin, N, H * Dh))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_deterministic(dtype):
    q, k, v = (t.to(dtype).cuda() for t in _qkv(4, 8, 144, 64))
    prec = P.BF16_MIXED if dtype == torch.bfloat16 else P.TF32_ACC_FP32
    a = fa.window_attn_fwd_cute(q, k, v, precision=prec)
    b = fa.window_attn_fwd_cute(q, k, v, precision=prec)
    assert torch.equal(a, b)


def test_dispatch_and_shape_limits():
    q, k, v = (t.cuda() for t in _qkv(4, 8, 64, 64))
    a = fa.window_attn_dispatch(q, k, v)
    assert a.dtype == torch.float32 and torch.equal(a, fa.window_attn_fwd_cute(q, k, v, precision=P.TF32_ACC_FP32))
    with pytest.raises(ValueError, match="144"):
        qq = torch.zeros(1, 1, 288, 64, device="cuda", dtype=torch.bfloat16)
        fa.window_attn_fwd_cute(qq, qq, qq)
    with pytest.raises(ValueError, match="head_dim"):
        qq = torch.zeros(1, 1, 144, 32, device="cuda", dtype=torch.bfloat16)
        fa.window_attn_fwd_cute(qq, qq, qq)
    empty = torch.zeros(0, 8, 144, 64, device="cuda", dtype=torch.bfloat16)
    assert fa.window_attn_fwd_cute(empty, empty, empty).shape == empty.shape


def test_non_contiguous_strided_inputs():
    Bwin, H, N, Dh = 5, 4, 144, 64
    base = torch.randn(Bwin, N, H, Dh * 2, device="cuda").bfloat16()
    q = base[..., :Dh].permute(0, 2, 1, 3)  # strided token/head, unit head-dim stride
    k = base[..., Dh:].permute(0, 2, 1, 3)
    v = base[..., :Dh].permute(0, 2, 1, 3)
    a = fa.window_attn_fwd_cute(q, k, v)
    b = fa.window_attn_fwd_cute(q.contiguous(), k.contiguous(), v.contiguous())
    assert torch.equal(a, b)


def test_status_word_clean_after_launches():
    from flash_aurora_b200 import _lib
    import ctypes
    st = ctypes.c_int(-1)
    _lib.check(_lib.load().fa_attention_status(ctypes.byref(st)), "status")
    assert st.value == 0


@pytest.mark.parametrize("has_mask", [False, True])
@pytest.mark.parametrize("N", [144, 96, 130])
def test_tensor_memory_kernel_matches_warp_mma_kernel(monkeypatch, has_mask, N):
    # The bf16 default is the tcgen05 kernel; FA_ATTN_BF16_KERNEL=mma_sync selects the warp-level
    # kernel. Both must agree to bf16 rounding on the same inputs.
    Bwin, H = 12, 4
    q, k, v = (t.bfloat16().cuda() for t in _qkv(Bwin, H, N, 64, seed=9, scale=1.0))
    bias = _half_bias(3, N).cuda() if has_mask else None
    a = fa.window_attn_fwd_cute(q, k, v, bias)
    monkeypatch.setenv("FA_ATTN_BF16_KERNEL", "mma_sync")
    b = fa.window_attn_fwd_cute(q, k, v, bias)
    monkeypatch.delenv("FA_ATTN_BF16_KERNEL")
    ref = OB.window_attention_core(q.double().cpu(), k.double().cpu(), v.double().cpu(),
                                   bias.double().cpu() if bias is not None else None)
    assert _rel_l2(a, ref) <= 1e-2 and _rel_l2(b, ref) <= 1e-2
    assert (a.float() - b.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("H", [1, 3, 8])
def test_region_id_patterns_all_mask_modes(H):
    """Arbitrary per-window region ids: one region (no mask), 2..16 distinct ids below 32 (mask
    UMMA), more than 16 distinct ids or ids >= 32 (per-logit fallback), in one launch."""
    N, nW = 144, 7
    g = torch.Generator().manual_seed(H)
    ids = torch.zeros(nW, N, dtype=torch.uint8)
    ids[0] = 4                                                   # one region
    ids[1] = torch.where(torch.arange(N) < 50, 5, 9).to(torch.uint8)       # two regions
    ids[2] = torch.randint(0, 16, (N,), generator=g).to(torch.uint8)      # up to 16 regions
    ids[3] = torch.randint(0, 17, (N,), generator=g).to(torch.uint8)      # 17 regions: fallback
    ids[4] = torch.randint(30, 42, (N,), generator=g).to(torch.uint8)     # ids >= 32: fallback
    ids[5] = torch.where(torch.arange(N) % 3 == 0, 0, 31).to(torch.uint8)  # ids 0 and 31
    ids[6] = torch.randint(0, 32, (N,), generator=g).to(torch.uint8)      # many regions: fallback
    bias = torch.where(ids[:, :, None] != ids[:, None, :], -100.0, 0.0)
    Bwin = 2 * nW
    q, k, v = _qkv(Bwin, H, N, 64, seed=11, scale=1.0)
    qc, kc, vc = (t.bfloat16().cuda() for t in (q, k, v))
    a = fa.window_attn_fwd_cute(qc, kc, vc, precision=P.BF16_MIXED, group_ids=ids.cuda())
    b = fa.window_attn_fwd_cute(qc, kc, vc, bias.cuda(), precision=P.BF16_MIXED)
    ref = OB.window_attention_core(*(t.bfloat16().double() for t in (q, k, v)), bias.double())
    for w in range(Bwin):
        assert _rel_l2(a[w], ref[w]) <= 1e-2, w
    assert (a.float() - b.float()).abs().max().item() <= 2e-2


def test_region_fit_flag_fast_path_and_broken_promise():
    """Region ids tagged as fitting the tensor-core mask run the kernel without the per-logit
    path; a tagged tensor that breaks the promise is reported through the status word (28)."""
    import ctypes

    from flash_aurora_b200 import _lib
    from flash_aurora_b200.window_attn import mark_region_ids_fit, region_ids_fit

    N, nW, H = 144, 4, 4
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 6, (nW, N), generator=g).to(torch.uint8)
    assert region_ids_fit(ids.numpy())
    q, k, v = (t.bfloat16().cuda() for t in _qkv(2 * nW, H, N, 64, seed=21, scale=1.0))
    plain = fa.window_attn_fwd_cute(q, k, v, group_ids=ids.cuda())            # fallback-capable kernel
    tagged = fa.window_attn_fwd_cute(q, k, v, group_ids=mark_region_ids_fit(ids.cuda()))
    assert torch.equal(plain, tagged)
    lib = _lib.load()
    _lib.check(lib.fa_attention_status_reset(None), "status reset")
    bad = torch.randint(0, 40, (nW, N), generator=g).to(torch.uint8)
    assert not region_ids_fit(bad.numpy())
    fa.window_attn_fwd_cute(q, k, v, group_ids=mark_region_ids_fit(bad.cuda()))
    torch.cuda.synchronize()
    st = ctypes.c_int(-1)
    _lib.check(lib.fa_attention_status(ctypes.byref(st)), "status")
    assert st.value == 28
    _lib.check(lib.fa_attention_status_reset(None), "status reset")


@pytest.mark.parametrize("mask", ["none", "bias", "groups"])
@pytest.mark.parametrize("N", [144, 130, 96])
def test_fp32_tensor_memory_kernel_matches_warp_mma_kernel(monkeypatch, mask, N):
    """FP32 I/O: the tcgen05 3xTF32 kernel (default) and the warp-level 3xTF32 kernel
    (FA_ATTN_FP32_KERNEL=mma_sync) both stay within the FP32-tier bound of strict FP64 attention.
    720 (window, head) tiles, so every CTA runs several tiles through its pipeline."""
    Bwin, H, nW = 90, 8, 6
    q, k, v = _qkv(Bwin, H, N, 64, seed=13, scale=0.5)
    g = torch.Generator().manual_seed(N)
    ids = torch.randint(0, 5, (nW, N), generator=g).to(torch.uint8)
    ids[0] = 2  # one region: nothing masked in this window
    bias = None
    kw = {}
    if mask == "bias":
        bias = _half_bias(nW, N)
        kw["bias"] = bias.cuda()
    elif mask == "groups":
        bias = torch.where(ids[:, :, None] != ids[:, None, :], -100.0, 0.0)
        kw["group_ids"] = ids.cuda()
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    a = fa.window_attn_fwd_cute(qc, kc, vc, precision=P.TF32_ACC_FP32, **kw)
    monkeypatch.setenv("FA_ATTN_FP32_KERNEL", "mma_sync")
    b = fa.window_attn_fwd_cute(qc, kc, vc, precision=P.TF32_ACC_FP32, **kw)
    monkeypatch.delenv("FA_ATTN_FP32_KERNEL")
    ref = OB.window_attention_core(q.double(), k.double(), v.double(),
                                   bias.double() if bias is not None else None)
    for out in (a, b):
        assert out.dtype == torch.float32
        assert _rel_l2(out, ref) <= 1e-5
        assert (out.cpu().double() - ref).abs().max().item() <= 2e-5
    assert (a - b).abs().max().item() <= 2e-5


@pytest.mark.parametrize("N", [144, 120])
def test_fp32_region_id_patterns_all_mask_modes(N):
    """FP32 I/O with region ids of many shapes in one launch (one region, 2..8 regions, 9 or more,
    ids >= 32, contiguous and scattered regions), against FP64 attention within the FP32-tier
    bound."""
    H, nW = 8, 8
    g = torch.Generator().manual_seed(N)
    ids = torch.zeros(nW, N, dtype=torch.uint8)
    ids[0] = 4                                                              # one region
    ids[1] = torch.where(torch.arange(N) < 50, 5, 9).to(torch.uint8)        # two regions
    ids[2] = torch.randint(0, 8, (N,), generator=g).to(torch.uint8)         # up to 8 regions
    ids[3] = (torch.arange(N) * 7 % 9).to(torch.uint8)                      # 9 regions: per logit
    ids[4] = torch.randint(30, 36, (N,), generator=g).to(torch.uint8)       # ids >= 32: per logit
    ids[5] = torch.where(torch.arange(N) % 3 == 0, 0, 31).to(torch.uint8)   # ids 0 and 31
    ids[6] = torch.randint(0, 24, (N,), generator=g).to(torch.uint8)        # many regions: per logit
    ids[7] = (torch.arange(N) // 18).to(torch.uint8)                        # 8 contiguous regions
    bias = torch.where(ids[:, :, None] != ids[:, None, :], -100.0, 0.0)
    Bwin = 3 * nW
    q, k, v = _qkv(Bwin, H, N, 64, seed=21, scale=0.5)
    a = fa.window_attn_fwd_cute(q.cuda(), k.cuda(), v.cuda(), precision=P.TF32_ACC_FP32, group_ids=ids.cuda())
    ref = OB.window_attention_core(q.double(), k.double(), v.double(), bias.double())
    for w in range(Bwin):
        assert _rel_l2(a[w], ref[w]) <= 1e-5, w
    assert (a.cpu().double() - ref).abs().max().item() <= 2e-5
