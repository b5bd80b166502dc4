"""The fused linear + AdaLN + residual kernel (``fa_linear_adaln_film``) against the unfused pair
(``linear_bias_act`` then the matching AdaLN op). The linear's output is rounded to bf16 exactly as
in the pair; the row statistics are fp32 two-pass in another summation order, so fp32 outputs agree
to 2e-6 (relative and absolute) and bf16 outputs to one bf16 ulp on at most 0.1 % of the elements.
Both row kinds, padded and unpadded window grids, batch 2, and M tails where the odd CTA of the
last pair has no rows; plus the block with the fusion on and off."""

from __future__ import annotations

import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200 import swin3d as S
from flash_aurora_b200.adaln import adaptive_layernorm_film_add_residual_partition
from flash_aurora_b200.linear import linear_adaln_film_add_residual, linear_bias_act

pytestmark = pytest.mark.gpu
WS = (2, 6, 12)


def _close_f32(got, want):
    torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)


def _close_bf16(got, want):
    """bf16 copies of fp32 values that agree to 2e-6: a rounding boundary between the two values
    moves the result by one bf16 ulp (at most 2^-7 of the value), plus the fp32 difference."""
    g, w = got.float(), want.float()
    diff = (g - w).abs()
    bound = w.abs() * 2 ** -7 + 4e-6
    assert bool((diff <= bound).all()), float((diff / bound).max())
    assert (diff > 0).float().mean().item() <= 1e-3


def _mod(B, D, g):
    return (torch.randn(B, 1, D, generator=g) * 0.1).cuda(), (torch.randn(B, 1, D, generator=g) * 0.1).cuda()


@pytest.mark.parametrize("res,shift,B", [((4, 36, 72), (1, 3, 6), 1), ((4, 45, 90), (1, 3, 6), 1),
                                         ((4, 45, 90), (0, 0, 0), 2), ((2, 12, 24), (1, 3, 6), 1)])
def test_windows_rows_equal_proj_then_unmerge_adaln(res, shift, B):
    g = torch.Generator().manual_seed(sum(res) + B)
    C, H, W = res
    L, D, K = C * H * W, 512, 512
    _, _, _, _, nW, N = fa.window_geometry(res, WS, shift)
    a = torch.randn(B * nW, N, K, generator=g).bfloat16().cuda()
    w = (torch.randn(D, K, generator=g) * 0.03).bfloat16().cuda()
    b = (torch.randn(D, generator=g) * 0.1).bfloat16().cuda()
    x = torch.randn(B, L, D, generator=g).cuda()
    sc, sh = _mod(B, D, g)
    want_bf = torch.empty(B, L, D, device="cuda", dtype=torch.bfloat16)
    proj = linear_bias_act(a, w, b, act="none")
    want = fa.unmerge_adaptive_layernorm_film_add_residual(proj, x, sc, sh, res, WS, shift, 0.0, 1e-5,
                                                           out_bf16=want_bf)
    got_bf = torch.empty_like(want_bf)
    got = linear_adaln_film_add_residual(a, w, b, x, sc, sh, res, WS, shift, rows="windows", out_bf16=got_bf)
    fa.check_device_status()
    _close_f32(got, want)
    _close_bf16(got_bf, want_bf)


@pytest.mark.parametrize("res,next_shift,K", [((4, 36, 72), (1, 3, 6), 2048), ((4, 45, 90), (0, 0, 0), 2048),
                                              ((4, 45, 90), None, 1024), ((2, 6, 12), (1, 3, 6), 64)])
def test_token_rows_equal_fc2_then_adaln(res, next_shift, K):
    g = torch.Generator().manual_seed(K + res[1])
    C, H, W = res
    L, D = C * H * W, 512
    h = torch.randn(1, L, K, generator=g).bfloat16().cuda()
    w = (torch.randn(D, K, generator=g) * 0.02).bfloat16().cuda()
    b = (torch.randn(D, generator=g) * 0.1).bfloat16().cuda()
    x1 = torch.randn(1, L, D, generator=g).cuda()
    sc, sh = _mod(1, D, g)
    y = linear_bias_act(h, w, b, act="none")
    if next_shift is None:
        want = fa.adaptive_layernorm_film_add_residual_forward(x1, y, sc, sh, 0.0, 1e-5, output_fp32=True)
        got = linear_adaln_film_add_residual(h, w, b, x1, sc, sh, res, WS, (0, 0, 0), rows="tokens")
    else:
        _, _, _, _, nW, N = fa.window_geometry(res, WS, next_shift)
        wb_want = torch.zeros(nW, N, D, device="cuda", dtype=torch.bfloat16)
        wb_got = torch.zeros_like(wb_want)
        want = adaptive_layernorm_film_add_residual_partition(x1, y, sc, sh, res, WS, next_shift, wb_want)
        got = linear_adaln_film_add_residual(h, w, b, x1, sc, sh, res, WS, (0, 0, 0), rows="tokens",
                                             next_windows=(next_shift, wb_got))
        _close_bf16(wb_got, wb_want)
    fa.check_device_status()
    _close_f32(got, want)


@pytest.mark.parametrize("flag", ["FUSE_FC2_ADALN", "FUSE_PROJ_ADALN"])
@pytest.mark.parametrize("shift", [(0, 0, 0), (1, 3, 6)])
def test_block_with_and_without_the_fusion(shift, flag, monkeypatch):
    """Each fused form of the block (fc2 -> norm2 is on by default, proj -> norm1 off) against the
    split path."""
    torch.manual_seed(9)
    res = (4, 24, 48)
    blk = S.Swin3DTransformerBlock(dim=512, num_heads=8, time_dim=512, window_size=WS, shift_size=shift)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0.0, 0.02)
    blk = blk.cuda().eval()
    g = torch.Generator().manual_seed(10)
    x = torch.randn(1, 4 * 24 * 48, 512, generator=g).cuda()
    c = torch.randn(1, 512, generator=g).cuda()
    with torch.no_grad():
        monkeypatch.setattr(S, "FUSE_FC2_ADALN", False)
        monkeypatch.setattr(S, "FUSE_PROJ_ADALN", False)
        split = blk(x, c, res)
        monkeypatch.setattr(S, flag, True)
        fused = blk(x, c, res)
    # norm1's output feeds fc1 through its bf16 copy, so a 1-ulp bf16 difference there reaches
    # norm2: compare the block outputs in relative L2 (the bf16 tier's own drift is ~1e-3).
    rel = ((fused - split).norm() / split.norm()).item()
    assert rel <= 5e-5, rel


def test_rejects_bad_arguments():
    a = torch.zeros(10, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(512, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(512, device="cuda", dtype=torch.bfloat16)
    x = torch.zeros(1, 4 * 6 * 12, 512, device="cuda")
    sc = torch.zeros(1, 1, 512, device="cuda")
    with pytest.raises(ValueError, match="M must be"):  # 10 rows for a 288-token grid
        linear_adaln_film_add_residual(a, w, b, x, sc, sc, (4, 6, 12), WS, (0, 0, 0), rows="tokens")
    with pytest.raises(ValueError, match="512 output"):
        linear_adaln_film_add_residual(a, w[:256], b[:256], x, sc, sc, (4, 6, 12), WS, (0, 0, 0), rows="tokens")
    with pytest.raises(ValueError, match="rows"):
        linear_adaln_film_add_residual(a, w, b, x, sc, sc, (4, 6, 12), WS, (0, 0, 0), rows="cols")
