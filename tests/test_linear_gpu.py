"""GPU parity of the tensor-core linear layer with the fused bias + GELU epilogue.

Reference: the same bf16 operands in float64 on the CPU (exact products, exact GELU). The fused
kernel rounds once (after the GELU); the unfused cuBLAS + GELU path rounds before and after, so the
fused result must be at least as close to the reference. Bounds: max error <= 1 bf16 ulp of the
largest output plus the fp32 accumulation error."""

from __future__ import annotations

import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

from flash_aurora_b200 import _lib
from flash_aurora_b200.linear import linear_bias_act

pytestmark = pytest.mark.gpu


def _ref(x, w, b, act):
    y = x.double().cpu() @ w.double().cpu().T + b.double().cpu()
    if act == "gelu":
        y = 0.5 * y * (1.0 + torch.erf(y / math.sqrt(2.0)))
    return y


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1000, 512, 512), (4099, 2048, 512), (259, 1536, 1024),
                                   (16200, 768, 128), (300, 256, 2048), (64, 512, 1024)])
@pytest.mark.parametrize("act", ["gelu", "none"])
@pytest.mark.parametrize("kernel", ["single", "pair"])
def test_linear_bias_act_matches_float64(M, N, K, act, kernel, monkeypatch):
    """Both kernels (single CTA, 128 x 256 tiles; CTA pair, 256 x 256 tiles), including M tails
    that leave the odd CTA of the last pair without a single row."""
    monkeypatch.setenv("FA_GEMM_KERNEL", kernel)
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16().cuda()
    b = (torch.randn(N, generator=g) * 0.1).bfloat16().cuda()
    got = linear_bias_act(x, w, b, act=act).cpu().double()
    ref = _ref(x, w, b, act)
    unfused = F.linear(x, w, b)
    if act == "gelu":
        unfused = F.gelu(unfused)
    unfused = unfused.cpu().double()
    err = (got - ref).abs()
    scale = ref.abs().max().item()
    assert err.max().item() <= scale * 2 ** -8 + 1e-3
    rel = (err.norm() / ref.norm()).item()
    rel_unfused = ((unfused - ref).norm() / ref.norm()).item()
    assert rel <= max(rel_unfused * 1.05, 2e-3)
    st = ctypes.c_int(-1)
    _lib.check(_lib.load().fa_gemm_status(ctypes.byref(st)), "status")
    assert st.value == 0


@pytest.mark.parametrize("M,N,K", [(259200, 2048, 512), (64800, 4096, 1024), (16200, 8192, 2048)])
def test_pair_and_single_kernels_agree_at_config4_shapes(M, N, K, monkeypatch):
    """At the config-4 fc1 shapes the two kernels accumulate the same products in the same K
    order (16-wide UMMA steps), so their outputs are identical."""
    g = torch.Generator(device="cuda").manual_seed(K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    b = (torch.randn(N, device="cuda", generator=g) * 0.02).bfloat16()
    outs = []
    for kernel in ("single", "pair"):
        monkeypatch.setenv("FA_GEMM_KERNEL", kernel)
        outs.append(linear_bias_act(x, w, b, act="gelu"))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("kernel", ["single", "pair"])
def test_gelu_epilogue_over_the_bf16_range(kernel, monkeypatch):
    """The epilogue's GELU on every finite bf16 value of magnitude up to 64: a 0/1 weight matrix
    routes each input value unchanged to one output element, so the epilogue sees exactly that
    value. Each result is the exact GELU rounded to bf16 or one bf16 unit away from it (rarely);
    below x = -7 (|GELU| < 1e-10) the fitted q overestimates the exact one, so there the bound is an
    absolute 1e-6, as for the standalone kernel's tail; results below the fp32 normal range
    (denormal inputs, or x * Phi(x) under 2^-126) may flush to zero."""
    monkeypatch.setenv("FA_GEMM_KERNEL", kernel)
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    vals = bits[torch.isfinite(bits.float()) & (bits.float().abs() <= 64)]
    K, N = 64, 256
    M = -(-vals.numel() // K)
    x = torch.zeros(M * K, dtype=torch.bfloat16)
    x[: vals.numel()] = vals
    x = x.view(M, K).cuda()
    w = torch.zeros(N, K, dtype=torch.bfloat16)
    w[torch.arange(N), torch.arange(N) % K] = 1
    b = torch.zeros(N, dtype=torch.bfloat16)
    got = linear_bias_act(x, w.cuda(), b.cuda(), act="gelu").cpu()
    inp = x.cpu().double()[:, torch.arange(N) % K]
    exact = 0.5 * inp * (1.0 + torch.erf(inp / math.sqrt(2.0)))
    want = exact.float().bfloat16()
    same = got == want
    # one bf16 unit: the spacing at the rounded exact value
    ulp = (want.float().abs() * 2.0 ** -7).clamp_min(2.0 ** -133)
    near = (got.float() - want.float()).abs() <= ulp * 1.01
    tail = (inp < -7) & ((got.double() - exact).abs() <= 1e-6)
    tiny = (exact.abs() < 2.0 ** -125) & (got.float().abs() <= 2.0 ** -125)
    assert (near | tail | tiny).all()
    body = (inp >= -7) & (exact.abs() >= 2.0 ** -125)
    assert (~same[body]).float().mean().item() < 2e-3


def test_linear_bias_act_batched_input_and_strided_rows():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 50, 640, generator=g).bfloat16().cuda()[..., :512]  # row stride 640
    w = (torch.randn(256, 512, generator=g) * 0.05).bfloat16().cuda()
    b = torch.zeros(256).bfloat16().cuda()
    got = linear_bias_act(x, w, b)
    assert got.shape == (3, 50, 256)
    ref = _ref(x.reshape(-1, 512), w, b, "gelu").reshape(3, 50, 256)
    assert (got.cpu().double() - ref).abs().max().item() <= ref.abs().max().item() * 2 ** -8 + 1e-3


def test_linear_bias_act_rejects_bad_shapes_and_status_clean():
    import ctypes
    x = torch.randn(10, 64).bfloat16().cuda()
    with pytest.raises(ValueError):
        linear_bias_act(x, torch.randn(100, 64).bfloat16().cuda(), torch.zeros(100).bfloat16().cuda())
    with pytest.raises(ValueError):
        linear_bias_act(x.float(), torch.randn(256, 64).cuda(), torch.zeros(256).cuda())
    linear_bias_act(x, torch.randn(256, 64).bfloat16().cuda(), torch.zeros(256).bfloat16().cuda())
    torch.cuda.synchronize()
    st = ctypes.c_int(-1)
    _lib.check(_lib.load().fa_gemm_status(ctypes.byref(st)), "status")
    assert st.value == 0
