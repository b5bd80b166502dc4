"""GPU parity of the exact-GELU kernel against PyTorch's CUDA GELU (the upstream nn.GELU())."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import flash_aurora_b200 as fa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 4099, 1_000_003, 2048 * 4096])
def test_gelu_matches_torch(dtype, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(n, device="cuda", generator=g) * 3).to(dtype)
    want = F.gelu(x)
    got = fa.gelu_erf(x)
    assert torch.equal(got, want)
    y = x.clone()
    fa.gelu_erf(y, inplace=True)
    assert torch.equal(y, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gelu_special_values_and_unaligned(dtype):
    vals = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e30, -1e30, float("inf"), float("-inf"), 3.0, -3.0,
                         -5.5, 10.0, -10.0, 0.5, -0.5], device="cuda").to(dtype)
    want = F.gelu(vals)
    got = fa.gelu_erf(vals)
    # GELU(-inf) = -inf * 0 is NaN in both; compare bits with NaN == NaN.
    torch.testing.assert_close(got, want, rtol=0, atol=0, equal_nan=True)
    nan = fa.gelu_erf(torch.tensor([float("nan")], device="cuda").to(dtype))
    assert torch.isnan(nan).all()
    base = torch.randn(10_001, device="cuda").to(dtype)
    x = base[1:]  # 2- or 4-byte offset: the scalar path
    assert torch.equal(fa.gelu_erf(x), F.gelu(x))


def test_gelu_rejects_partial_overlap():
    x = torch.randn(1024, device="cuda", dtype=torch.bfloat16)
    from flash_aurora_b200 import _lib
    rc = _lib.load().fa_gelu_erf(x.data_ptr(), x[8:].data_ptr(), _lib.FA_BF16, 512, None)
    assert rc == _lib.FA_ERR_INVALID
