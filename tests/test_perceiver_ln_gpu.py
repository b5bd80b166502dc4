"""GPU parity of the Perceiver decoder LayerNorm (+ residual) kernel, fa_layernorm_affine.

Upstream's own checks (tests/kernels/test_triton_perceiver_ln.py:12-38: (2, 31, 256), against
nn.LayerNorm in the same dtype, rtol = atol = 1e-5 for fp32 and 2e-2 for bf16) plus a tighter one:
against the fused semantics computed in float64 and rounded once to the output dtype, the kernel
is within 2e-6 relative (fp32) or two units in the last place (bf16 / fp16, plus 1e-5 absolute
near zero)."""

from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn as nn

import flash_aurora_b200 as fa
from flash_aurora_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm_affine_matches_module(dtype):
    B, L, D = 2, 31, 256
    torch.manual_seed(0)
    x = torch.randn(B, L, D, device="cuda", dtype=dtype)
    ln = nn.LayerNorm(D).to(device="cuda", dtype=dtype)
    with torch.no_grad():
        ln.weight.normal_(1.0, 0.2)
        ln.bias.normal_(0.0, 0.2)
    ref = ln(x)
    got = fa.layernorm_affine_forward(x, ln.weight, ln.bias, float(ln.eps))
    rtol, atol = (2e-2, 2e-2) if dtype == torch.bfloat16 else (1e-5, 1e-5)
    assert got.dtype == dtype and got.shape == x.shape
    torch.testing.assert_close(ref, got, rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm_affine_add_residual_matches_torch(dtype):
    B, L, D = 2, 31, 256
    torch.manual_seed(1)
    x = torch.randn(B, L, D, device="cuda", dtype=dtype)
    residual = torch.randn(B, L, D, device="cuda", dtype=dtype)
    ln = nn.LayerNorm(D).to(device="cuda", dtype=dtype)
    ref = ln(x) + residual
    got = fa.layernorm_affine_add_residual_forward(x, residual, ln.weight, ln.bias, float(ln.eps))
    rtol, atol = (2e-2, 2e-2) if dtype == torch.bfloat16 else (1e-5, 1e-5)
    torch.testing.assert_close(ref, got, rtol=rtol, atol=atol)


def _fused_ref(x, w, b, eps, r=None):
    x64 = x.double()
    mean = x64.mean(-1, keepdim=True)
    var = ((x64 - mean) ** 2).mean(-1, keepdim=True)
    y = (x64 - mean) / torch.sqrt(var + eps) * w.double() + b.double()
    if r is not None:
        y = y + r.double()
    return y


def _check_one_rounding(got, y64):
    if got.dtype == torch.float32:
        err = (got.double() - y64).abs()
        assert (err <= 2e-6 * y64.abs() + 2e-6).all(), err.max().item()
        return
    # within one ulp of the float64 result in the output format
    ulp = torch.finfo(got.dtype).eps * torch.maximum(y64.abs(), torch.full_like(y64, torch.finfo(got.dtype).tiny))
    ulp = 2.0 ** torch.floor(torch.log2(ulp))
    err = (got.double() - y64).abs()
    # 1.5 ulp covers the fp32 arithmetic moving a value across a rounding boundary; the absolute
    # term covers outputs near zero, where that fp32 error exceeds their ulp.
    assert (err <= 2 * ulp + 1e-5).all(), (err / ulp).max().item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [1, 100, 256, 512, 1000, 2048, 4096])
@pytest.mark.parametrize("residual", [False, True])
def test_fused_semantics_one_rounding(dtype, D, residual):
    torch.manual_seed(D)
    rows = 37
    x = (torch.randn(1, rows, D, device="cuda") * 3 + 1).to(dtype)
    w = torch.randn(D, device="cuda").to(dtype)
    b = torch.randn(D, device="cuda").to(dtype)
    r = torch.randn(1, rows, D, device="cuda").to(dtype) if residual else None
    got = (fa.layernorm_affine_add_residual_forward(x, r, w, b, 1e-5) if residual
           else fa.layernorm_affine_forward(x, w, b, 1e-5))
    _check_one_rounding(got, _fused_ref(x, w, b, 1e-5, r))


def test_mixed_parameter_dtype_and_decoder_shape():
    """bf16 activations with fp32 LayerNorm parameters, at a slice of the era5 level-decoder shape
    (latents (B*H*W, 13 levels, 512))."""
    torch.manual_seed(3)
    x = torch.randn(4096, 13, 512, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(512, device="cuda") * 0.5 + 1
    b = torch.randn(512, device="cuda") * 0.1
    got = fa.layernorm_affine_add_residual_forward(x, r, w, b, 1e-5)
    _check_one_rounding(got, _fused_ref(x, w, b, 1e-5, r))


def test_unaligned_rows_and_in_place_through_the_c_abi():
    lib = _lib.load()
    torch.manual_seed(4)
    D, rows = 256, 9
    buf = torch.randn(rows * D + 1, device="cuda")
    x = buf[1:]  # 4-byte offset: the scalar path
    w = torch.randn(D, device="cuda")
    b = torch.randn(D, device="cuda")
    y64 = _fused_ref(x.view(rows, D), w, b, 1e-5)
    out = torch.empty(rows * D + 1, device="cuda")[1:]
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.fa_layernorm_affine(x.data_ptr(), _lib.FA_F32, None, w.data_ptr(), b.data_ptr(), _lib.FA_F32,
                                       1e-5, out.data_ptr(), rows, D, s), "ln")
    _check_one_rounding(out.view(rows, D), y64)
    # in place (aligned): out aliases x
    xa = x.clone()
    _lib.check(lib.fa_layernorm_affine(xa.data_ptr(), _lib.FA_F32, None, w.data_ptr(), b.data_ptr(), _lib.FA_F32,
                                       1e-5, xa.data_ptr(), rows, D, s), "ln")
    _check_one_rounding(xa.view(rows, D), y64)


def test_empty_and_limits():
    x = torch.empty(0, 5, 64, device="cuda")
    assert fa.layernorm_affine_forward(x, torch.ones(64, device="cuda"), torch.zeros(64, device="cuda"), 1e-5).shape == x.shape
    with pytest.raises(ValueError, match="4096"):
        fa.layernorm_affine_forward(torch.zeros(1, 1, 4097, device="cuda"), torch.ones(4097, device="cuda"),
                                    torch.zeros(4097, device="cuda"), 1e-5)
    with pytest.raises(ValueError, match="Unsupported dtype"):
        fa.layernorm_affine_forward(torch.zeros(1, 1, 8, device="cuda", dtype=torch.float64),
                                    torch.ones(8, device="cuda"), torch.zeros(8, device="cuda"), 1e-5)
