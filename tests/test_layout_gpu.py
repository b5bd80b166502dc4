"""GPU parity of the fused window layout: bit-exact against the oracle index maps (which are
pinned to the upstream fixtures), for every golden geometry, both dtypes, vector and scalar
paths, plus round trips at the full config-3 size."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flash_aurora_b200 as fa
from oracle import layout as OL

pytestmark = pytest.mark.gpu

PAIRS = [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
         (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)]


def _cases(golden):
    d = golden("layout_maps.npz")
    out = []
    for name in sorted({k.split("/")[0] for k in d if k.endswith("/spec")}):
        s = [int(a) for a in d[f"{name}/spec"]]
        out.append((name, tuple(s[:3]), tuple(s[3:6]), tuple(s[6:9])))
    return out


@pytest.mark.parametrize("din,dout", PAIRS)
@pytest.mark.parametrize("D", [32, 5])
def test_partition_and_unmerge_bit_exact(golden, din, dout, D):
    g = torch.Generator().manual_seed(0)
    for name, res, ws, ss in _cases(golden):
        x = torch.randn(2, *res, D, generator=g).to(din)
        ref = OL.roll_pad_partition(x.float().numpy(), res, ws, ss)
        ref = torch.from_numpy(ref).to(dout)
        got = fa.roll_pad_partition_windows_triton(x.cuda(), res, ws, ss, out_dtype=dout).cpu()
        assert got.dtype == dout
        assert torch.equal(got, ref), name
        w = torch.randn(*ref.shape, generator=g).to(din)
        ref_u = torch.from_numpy(OL.crop_roll_unmerge(w.float().numpy(), res, ws, ss)).to(dout)
        got_u = fa.crop_roll_unmerge_windows_triton(w.cuda(), res, ws, ss, out_dtype=dout).cpu()
        assert torch.equal(got_u, ref_u), name


def test_upstream_test_shapes_roundtrip():
    # Upstream test_triton_swin3d.py:120-134: B=1, (4,8,16), D=64, ws (2,4,4), ss (1,2,2).
    x = torch.randn(1, 4, 8, 16, 64, device="cuda")
    w = fa.roll_pad_partition_windows_triton(x, (4, 8, 16), (2, 4, 4), (1, 2, 2))
    back = fa.crop_roll_unmerge_windows_triton(w, (4, 8, 16), (2, 4, 4), (1, 2, 2))
    assert torch.equal(back, x)


@pytest.mark.parametrize("D", [2048, 512])
def test_config3_full_size_roundtrip(D):
    # Config 3: grid (4,45,90), dim 2048, padded to (4,48,96), 128 windows, shift (1,3,6).
    res, ws, ss = (4, 45, 90), (2, 6, 12), (1, 3, 6)
    x = torch.randn(1, *res, D, device="cuda")
    for shift in (ss, (0, 0, 0)):
        w = fa.roll_pad_partition_windows(x, res, ws, shift)
        assert w.shape == (128, 144, D)
        back = fa.crop_roll_unmerge_windows(w, res, ws, shift)
        assert torch.equal(back, x)
        # Pad tokens are exact zeros and every input row appears exactly once.
        src = OL.partition_source_index(OL.geometry(res, ws, shift))
        pad = torch.from_numpy(src.reshape(-1) < 0).cuda()
        assert torch.count_nonzero(w.reshape(-1, D)[pad]) == 0
        assert int((~pad).sum()) == 4 * 45 * 90
    wb = fa.roll_pad_partition_windows(x, res, ws, ss, out_dtype=torch.bfloat16)
    assert torch.equal(wb, fa.roll_pad_partition_windows(x.bfloat16(), res, ws, ss))


def test_pool_reuses_output():
    pool = fa.InferenceWorkspacePool()
    x = torch.randn(1, 4, 36, 72, 64, device="cuda")
    a = fa.roll_pad_partition_windows(x, (4, 36, 72), (2, 6, 12), (1, 3, 6), pool=pool)
    b = fa.roll_pad_partition_windows(x, (4, 36, 72), (2, 6, 12), (1, 3, 6), pool=pool)
    assert a.data_ptr() == b.data_ptr() and torch.equal(a, b)


def test_empty_batch():
    x = torch.empty(0, 4, 36, 72, 64, device="cuda")
    w = fa.roll_pad_partition_windows(x, (4, 36, 72), (2, 6, 12), (1, 3, 6))
    assert w.shape == (0, 144, 64)
