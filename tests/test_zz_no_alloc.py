"""The allocation-free attention entry point, for callers that cannot call cudaMalloc.

``fa_window_attention_bias_noalloc`` takes the float shifted-window bias and packs it into a
static device array of the library instead of a temporary buffer, so code running under a memory
pool it does not own, or in a loop that must not allocate, can still use the float-bias API.
These tests call it through the C ABI and compare it with ``fa_window_attention`` on two calls in
a row (the second call reuses the scratch left by the first). This file is collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200 import _lib
from oracle import block as OB

pytestmark = pytest.mark.gpu

MAX_MASK_BYTES = 4 << 20


def _noalloc(q, k, v, bias, precision, scale):
    out = torch.empty_like(q)
    strides = (ctypes.c_int64 * 12)(*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3])
    Bwin, H, N, Dh = q.shape
    rc = _lib.load().fa_window_attention_bias_noalloc(
        precision, Bwin, H, N, Dh, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), strides,
        bias.data_ptr(), bias.shape[0], float(scale), _lib.stream_ptr(q.device))
    _lib.check(rc, "fa_window_attention_bias_noalloc")
    return out


def _bias(nW, N, seed):
    g = torch.Generator().manual_seed(seed)
    groups = torch.randint(0, 3, (nW, N), generator=g)
    return torch.where(groups[:, None, :] != groups[:, :, None], -100.0, 0.0).float()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_allocating_entry_point_on_two_calls(dtype):
    Bwin, H, N, Dh, nW = 12, 8, 144, 64, 4
    g = torch.Generator().manual_seed(0)
    q, k, v = ((torch.randn(Bwin, H, N, Dh, generator=g)).to(dtype).cuda() for _ in range(3))
    prec = fa.WinAttnPrecision.BF16_MIXED if dtype == torch.bfloat16 else fa.WinAttnPrecision.TF32_ACC_FP32
    code = _lib.FA_ATTN_BF16 if dtype == torch.bfloat16 else _lib.FA_ATTN_FP32_3XTF32
    scale = Dh ** -0.5
    for call, seed in enumerate((1, 2)):  # second call: different mask, same scratch
        bias = _bias(nW, N, seed).cuda()
        want = fa.window_attn_fwd_cute(q, k, v, bias, scale_qk=scale, precision=prec)
        got = _noalloc(q, k, v, bias, code, scale)
        torch.cuda.synchronize()
        # Same kernel on the same packed mask: the two entry points agree bit for bit.
        assert torch.equal(got, want), f"call {call}"
        # And against the CPU restatement of the upstream attention, within the attention tests'
        # tolerance for this precision (relative L2).
        ref = OB.window_attention_core(q.float().cpu(), k.float().cpu(), v.float().cpu(), bias.cpu(), scale)
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
        assert OB.relative_l2(got.float().cpu(), ref) <= tol, f"call {call}"


def test_noalloc_checks_arguments_before_writing_the_scratch():
    """A call rejected for its shape returns the error and leaves the scratch alone: a valid call
    before and after it gives the same result."""
    Bwin, H, N, Dh, nW = 4, 2, 144, 64, 4
    g = torch.Generator().manual_seed(3)
    q, k, v = ((torch.randn(Bwin, H, N, Dh, generator=g)).bfloat16().cuda() for _ in range(3))
    bias = _bias(nW, N, 5).cuda()
    first = _noalloc(q, k, v, bias, _lib.FA_ATTN_BF16, 0.125)
    big = torch.zeros(1, 1, 160, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="N <= 144"):
        _noalloc(big, big, big, torch.full((1, 160, 160), -100.0, device="cuda"), _lib.FA_ATTN_BF16, 0.125)
    with pytest.raises(ValueError, match="head_dim"):
        odd = torch.zeros(1, 1, N, 32, device="cuda", dtype=torch.bfloat16)
        _noalloc(odd, odd, odd, bias, _lib.FA_ATTN_BF16, 0.125)
    again = _noalloc(q, k, v, bias, _lib.FA_ATTN_BF16, 0.125)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_noalloc_rejects_masks_beyond_the_static_scratch():
    N = 144
    nW = MAX_MASK_BYTES // (N * N) + 1
    q = torch.zeros(nW, 1, N, 64, device="cuda", dtype=torch.bfloat16)
    bias = torch.zeros(nW, N, N, device="cuda")
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(q, q, q, bias, _lib.FA_ATTN_BF16, 0.125)
