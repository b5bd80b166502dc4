"""GPU parity of the fused AdaLN (+ residual, + unmerge) against the oracle and the upstream
AdaptiveLayerNorm fixtures."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flash_aurora_b200 as fa
from oracle import block as OB
from oracle import layout as OL

pytestmark = pytest.mark.gpu


def test_matches_upstream_fixture(golden):
    d = golden("adaln.npz")
    for tag in ("d256", "d2048"):
        t = {k.split("/", 1)[1]: torch.from_numpy(v) for k, v in d.items() if k.startswith(tag + "/")}
        y = fa.adaptive_layernorm_film_forward(t["x"].cuda(), t["scale"].cuda(), t["shift"].cuda(), 0.0, 1e-5,
                                               output_fp32=True).cpu()
        torch.testing.assert_close(y, t["forward"], rtol=1e-5, atol=1e-5)
        xb = t["x_bf16_valued"].bfloat16().cuda()
        yr = fa.adaptive_layernorm_film_add_residual_forward(t["residual"].cuda(), xb, t["scale"].cuda(),
                                                             t["shift"].cuda(), 0.0, 1e-5, output_fp32=True).cpu()
        torch.testing.assert_close(yr, t["forward_add_residual"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("D", [128, 256, 512, 1024, 2048, 200, 37])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_add_residual_vs_oracle(D, xdt):
    g = torch.Generator().manual_seed(D)
    B, L = 2, 67
    x = torch.randn(B, L, D, generator=g).to(xdt)
    res = torch.randn(B, L, D, generator=g)
    scale = torch.randn(B, 1, D, generator=g) * 0.5
    shift = torch.randn(B, 1, D, generator=g) * 0.5
    ref = res + OB.adaln(x.float(), shift, scale, scale_bias=0.25)
    out_bf16 = torch.empty(B, L, D, dtype=torch.bfloat16, device="cuda")
    got = fa.adaptive_layernorm_film_add_residual_forward(res.cuda(), x.cuda(), scale.cuda(), shift.cuda(), 0.25,
                                                          output_fp32=True, out_bf16=out_bf16)
    torch.testing.assert_close(got.cpu(), ref, rtol=2e-5, atol=2e-5)
    assert torch.equal(out_bf16, got.bfloat16())


def test_output_dtypes_follow_upstream():
    x = torch.randn(2, 8, 64, device="cuda", dtype=torch.bfloat16)
    s = torch.randn(2, 1, 64, device="cuda")
    assert fa.adaptive_layernorm_film_forward(x, s, s, 0.0).dtype == torch.bfloat16
    assert fa.adaptive_layernorm_film_forward(x, s, s, 0.0, output_fp32=True).dtype == torch.float32
    with pytest.raises(ValueError, match="same dtype"):
        fa.adaptive_layernorm_film_add_residual_forward(torch.randn(2, 8, 64, device="cuda"), x, s, s, 0.0)
    with pytest.raises(ValueError, match="float32"):
        fa.adaptive_layernorm_film_add_residual_forward(x, x, s, s, 0.0, output_fp32=True)
    with pytest.raises(ValueError, match="2048"):
        fa.adaptive_layernorm_film_forward(torch.randn(1, 2, 4096, device="cuda"), torch.randn(1, 1, 4096, device="cuda"),
                                           torch.randn(1, 1, 4096, device="cuda"), 0.0)
    # bf16 in/out with bf16 residual (output_fp32=False).
    r = torch.randn(2, 8, 64, device="cuda", dtype=torch.bfloat16)
    y = fa.adaptive_layernorm_film_add_residual_forward(r, x, s, s, 0.0)
    ref = r.float() + OB.adaln(x.float().cpu(), s.cpu(), s.cpu()).cuda()
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("res,ws,ss", [((4, 36, 72), (2, 6, 12), (1, 3, 6)), ((4, 45, 90), (2, 6, 12), (1, 3, 6)),
                                       ((3, 13, 25), (2, 6, 12), (0, 0, 0))])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [256, 1024])
def test_unmerge_fused_equals_composition(res, ws, ss, wdt, D):
    g = torch.Generator().manual_seed(1)
    gm = OL.geometry(res, ws, ss)
    B = 2
    L = res[0] * res[1] * res[2]
    win = torch.randn(B * gm.num_windows, gm.window_tokens, D, generator=g).to(wdt).cuda()
    resid = torch.randn(B, L, D, generator=g).cuda()
    scale = torch.randn(B, 1, D, generator=g).cuda()
    shift = torch.randn(B, 1, D, generator=g).cuda()
    merged = fa.crop_roll_unmerge_windows(win, res, ws, ss).reshape(B, L, D)
    ref = fa.adaptive_layernorm_film_add_residual_forward(resid, merged.float(), scale, shift, 0.0, output_fp32=True)
    xb = torch.empty(B, L, D, dtype=torch.bfloat16, device="cuda")
    got = fa.unmerge_adaptive_layernorm_film_add_residual(win, resid, scale, shift, res, ws, ss, out_bf16=xb)
    assert torch.equal(got, ref)
    assert torch.equal(xb, ref.bfloat16())


@pytest.mark.parametrize("res,shift", [((4, 36, 72), (1, 3, 6)), ((4, 45, 90), (1, 3, 6)), ((4, 45, 90), (0, 0, 0))])
@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
def test_adaln_partition_fused_equals_adaln_then_partition(res, shift, wdtype):
    C, H, W = res
    D, ws = 128, (2, 6, 12)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, C * H * W, D, generator=g).bfloat16().cuda()
    resid = torch.randn(1, C * H * W, D, generator=g).cuda()
    scale = (torch.randn(1, 1, D, generator=g) * 0.1).cuda()
    shf = (torch.randn(1, 1, D, generator=g) * 0.1).cuda()
    want = fa.adaptive_layernorm_film_add_residual_forward(resid, x, scale, shf, 0.0, output_fp32=True)
    want_w = fa.roll_pad_partition_windows(want.view(1, C, H, W, D), res, ws, shift, out_dtype=wdtype)
    from flash_aurora_b200.adaln import adaptive_layernorm_film_add_residual_partition
    win = torch.zeros_like(want_w)
    got = adaptive_layernorm_film_add_residual_partition(resid, x, scale, shf, res, ws, shift, win)
    assert torch.equal(got, want)
    assert torch.equal(win, want_w)
