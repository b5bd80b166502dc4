"""Parity at the benchmarked attention size (config 2): the full stage-1 launch, 1800 windows of
grid (4,180,360) x 8 heads x N=144 x Dh=64, packed QKV ~N(0,1)/8, with the real shifted-window
region ids of that grid (930 of 1800 windows masked), against the CPU oracle (FP32 SDPA semantics
with upstream's -100 mask), computed in chunks of windows.

Bounds: bf16 I/O relative L2 <= 1e-2 (and the upstream elementwise 2e-2 bound); fp32 I/O
(3xTF32) relative L2 <= 1e-5."""

from __future__ import annotations

import pytest
import torch

import flash_aurora_b200 as fa
from oracle import block as OB

pytestmark = pytest.mark.gpu

RES, WS, SS = (4, 180, 360), (2, 6, 12), (1, 3, 6)
BWIN, H, N, DH = 1800, 8, 144, 64


def _oracle(qkv32: torch.Tensor, gids: torch.Tensor, chunk: int = 150) -> torch.Tensor:
    """(Bwin, N, H*Dh) attention output of the oracle for packed fp32 qkv on the CPU."""
    q, k, v = qkv32.view(BWIN, N, 3, H, DH).permute(2, 0, 3, 1, 4)
    out = torch.empty(BWIN, N, H * DH)
    for w0 in range(0, BWIN, chunk):
        sl = slice(w0, w0 + chunk)
        g = gids[sl].long()
        mask = torch.where(g[:, :, None] != g[:, None, :], -100.0, 0.0)
        o = OB.window_attention_core(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous(), mask)
        out[sl] = o.permute(0, 2, 1, 3).reshape(-1, N, H * DH)
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config2_full_launch_against_oracle(dtype):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    g = torch.Generator().manual_seed(2)
    qkv = (torch.randn(BWIN, N, 3 * H * DH, generator=g) / 8.0).to(dtype)
    gids_cpu = fa.shifted_window_group_ids(RES, WS, SS)
    assert gids_cpu.shape == (BWIN, N)
    masked = int((gids_cpu.amax(dim=1) != gids_cpu.amin(dim=1)).sum())
    assert masked == 930
    gids = fa.shifted_window_group_ids(RES, WS, SS, device=torch.device("cuda"))
    got = fa.window_attn_fwd_cute_qkvpacked(qkv.cuda(), H, group_ids=gids, output_layout="bnc")
    fa.check_device_status()
    ref = _oracle(qkv.float(), gids_cpu)
    got = got.float().cpu()
    rel = OB.relative_l2(got, ref)
    if dtype == torch.bfloat16:
        assert rel <= 1e-2, rel
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)
    else:
        assert rel <= 1e-5, rel
