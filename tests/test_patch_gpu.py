"""GPU parity of the fused stage-boundary kernels (patch merge + LayerNorm, patch split + LayerNorm)
against the upstream-order PyTorch formulation (pad / permute / crop, then LayerNorm) on the same
inputs, including odd H / W (merge padding) and crops (split)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from flash_aurora_b200.swin3d import PatchMerging3D, PatchSplitting3D

pytestmark = pytest.mark.gpu


def _merge_ref(m, x, res):
    C, H, W = res
    B, L, D = x.shape
    x = x.view(B, C, H, W, D)
    x = F.pad(x, (0, 0, 0, W % 2, 0, H % 2))
    nH, nW = x.shape[2], x.shape[3]
    x = x.reshape(B, C, nH // 2, 2, nW // 2, 2, D).permute(0, 1, 2, 4, 3, 5, 6).reshape(B, -1, 4 * D)
    return m.reduction(m.norm(x))


def _split_ref(m, x, res, crop):
    C, H, W = res
    x = m.lin1(x)
    B, L, D = x.shape
    x = x.view(B, C, H, W, 2, 2, D // 4).permute(0, 1, 2, 4, 3, 5, 6).reshape(B, C, 2 * H, 2 * W, D // 4)
    cC, cH, cW = crop
    x = x[:, : x.shape[1] - cC, : x.shape[2] - cH, : x.shape[3] - cW, :].reshape(B, -1, D // 4)
    return m.lin2(m.norm(x))


@pytest.mark.parametrize("res,D", [((4, 36, 72), 64), ((4, 45, 90), 128), ((2, 13, 25), 512), ((4, 6, 12), 1024)])
def test_patch_merge_fused_matches_reference(res, D):
    torch.manual_seed(0)
    m = PatchMerging3D(D).cuda()
    with torch.no_grad():
        m.norm.weight.normal_(1.0, 0.1)
        m.norm.bias.normal_(0.0, 0.1)
        C, H, W = res
        x = torch.randn(2, C * H * W, D, device="cuda")
        torch.backends.cuda.matmul.allow_tf32 = False
        got = m(x, res)
        want = _merge_ref(m, x, res)
    assert got.shape == want.shape
    torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("res,dim,crop", [((4, 18, 36), 128, (0, 0, 0)), ((4, 23, 45), 256, (0, 1, 0)),
                                          ((2, 12, 24), 2048, (0, 0, 0)), ((3, 5, 7), 64, (1, 1, 1))])
def test_patch_split_fused_matches_reference(res, dim, crop):
    torch.manual_seed(1)
    m = PatchSplitting3D(dim).cuda()
    with torch.no_grad():
        m.norm.weight.normal_(1.0, 0.1)
        m.norm.bias.normal_(0.0, 0.1)
        C, H, W = res
        x = torch.randn(1, C * H * W, dim, device="cuda")
        torch.backends.cuda.matmul.allow_tf32 = False
        got = m(x, res, crop)
        want = _split_ref(m, x, res, crop)
    assert got.shape == want.shape
    torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-5)
