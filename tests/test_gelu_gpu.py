"""GPU parity of the GELU kernel.

method "erff": bit-identical to PyTorch's CUDA GELU (the upstream nn.GELU()).
method "poly": every finite bf16 input is checked against the exact GELU computed in float64 on
the CPU and rounded to bf16: equal for |x| < 4, within 1e-6 beyond (where |GELU| < 1.3e-4)."""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import flash_aurora_b200 as fa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 4099, 1_000_003, 2048 * 4096])
def test_gelu_erff_matches_torch(dtype, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(n, device="cuda", generator=g) * 3).to(dtype)
    want = F.gelu(x)
    got = fa.gelu_erf(x, method="erff")
    assert torch.equal(got, want)
    y = x.clone()
    fa.gelu_erf(y, inplace=True, method="erff")
    assert torch.equal(y, want)


def _exact_gelu_f64(x: torch.Tensor) -> torch.Tensor:
    xd = x.double().cpu()
    return 0.5 * xd * (1.0 + torch.erf(xd / math.sqrt(2.0)))


def test_gelu_poly_every_bf16_input():
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    x = bits[torch.isfinite(bits.float())].cuda()
    got = fa.gelu_erf(x, method="poly").cpu()
    exact = _exact_gelu_f64(x)
    want = exact.float().bfloat16()
    inner = x.cpu().float().abs() < 4
    assert torch.equal(got[inner], want[inner])
    # |x| >= 4: the rounded exact value, or within 1e-6 of the exact value (the tiny x < -4 tail)
    ok = (got == want) | ((got.double() - exact).abs() <= 1e-6)
    assert ok[~inner].all()
    # in place, fp32 and the unaligned scalar path agree with the vector path
    y = x.clone()
    fa.gelu_erf(y, inplace=True)
    assert torch.equal(y.cpu(), got)
    base = torch.cat([x[:1], x])
    assert torch.equal(fa.gelu_erf(base[1:]).cpu(), got)


@pytest.mark.parametrize("n", [1, 4099, 1_000_003])
def test_gelu_poly_fp32_close_to_exact(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(n, device="cuda", generator=g) * 3
    got = fa.gelu_erf(x, method="poly").cpu().double()
    exact = _exact_gelu_f64(x)
    # |error| <= a few fp32 ulps of |x| (the erff form has the same order near the tails)
    assert ((got - exact).abs() <= 4e-7 * x.cpu().double().abs() + 1e-30).all()


@pytest.mark.parametrize("method", ["erff", "poly"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gelu_special_values(method, dtype):
    vals = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e30, -1e30, float("inf"), float("-inf"), 3.0, -3.0,
                         -5.5, 10.0, -10.0, 0.5, -0.5], device="cuda").to(dtype)
    got = fa.gelu_erf(vals, method=method)
    want = F.gelu(vals)
    if method == "erff":
        torch.testing.assert_close(got, want, rtol=0, atol=0, equal_nan=True)
    else:
        torch.testing.assert_close(got.float(), want.float(), rtol=8e-3, atol=1e-6, equal_nan=True)
    nan = fa.gelu_erf(torch.tensor([float("nan")], device="cuda").to(dtype), method=method)
    assert torch.isnan(nan).all()


def test_gelu_rejects_partial_overlap_and_bad_method():
    x = torch.randn(1024, device="cuda", dtype=torch.bfloat16)
    from flash_aurora_b200 import _lib
    rc = _lib.load().fa_gelu_erf(x.data_ptr(), x[8:].data_ptr(), _lib.FA_BF16, 512, _lib.FA_GELU_POLY, None)
    assert rc == _lib.FA_ERR_INVALID
    with pytest.raises(ValueError):
        fa.gelu_erf(x, method="tanh")
