"""GPU parity of the latitude-band kernels and of the sharded Swin3D block.

* band partition / halo extract / band unmerge / band unmerge+AdaLN against the whole-field
  kernels and the numpy oracle: bit-exact;
* a block stack run on emulated ranks (threads of one process sharing one GPU, halo exchanged
  through ``LocalRing``) against the unsharded stack on the whole field;
* with two or more GPUs, the same over NCCL with one process per GPU.
"""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200 import sharding
from flash_aurora_b200.swin3d import BasicLayer3D
from oracle import block as OB
from oracle import layout as L

pytestmark = pytest.mark.gpu

WS = (2, 6, 12)
SHIFT = (1, 3, 6)


def _x(field_res, D, dtype, seed=0, B=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((B,) + tuple(field_res) + (D,), generator=g).to(dtype).cuda()


@pytest.mark.parametrize("field_res,D", [((4, 36, 72), 64), ((3, 24, 30), 40), ((4, 12, 24), 36)])
@pytest.mark.parametrize("shift", [(0, 0, 0), SHIFT])
@pytest.mark.parametrize("dt_in,dt_out", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                          (torch.bfloat16, torch.bfloat16)])
def test_band_layout_bit_exact(field_res, D, shift, dt_in, dt_out):
    x = _x(field_res, D, dt_in, seed=D)
    wf = fa.roll_pad_partition_windows(x, field_res, WS, shift, out_dtype=dt_out)
    _, ss = L.maybe_adjust_windows(WS, shift, field_res)
    s = ss[1]
    H = field_res[1]
    rows = H // WS[1]
    for world in sorted({1, 2, min(3, rows), rows}):
        bands = sharding.band_bounds(field_res, WS, world)
        backs = {}
        for r, (a, b) in enumerate(bands):
            nb = bands[(r + 1) % world][0]
            halo = x[:, :, nb:nb + s].contiguous() if s else None
            wb = fa.roll_pad_partition_windows_band(x[:, :, a:b].contiguous(), halo, field_res, WS, shift,
                                                    out_dtype=dt_out)
            ref = L.band_windows_of_field(wf.cpu().float().numpy(), field_res, WS, shift, a, b)
            assert torch.equal(wb.cpu().float(), torch.from_numpy(ref)), (world, r)
            if s and dt_in != dt_out:
                # A halo sent already rounded to the windows' dtype gives the same windows.
                wb2 = fa.roll_pad_partition_windows_band(x[:, :, a:b].contiguous(), halo.to(dt_out), field_res, WS,
                                                         shift, out_dtype=dt_out)
                assert torch.equal(wb2, wb), (world, r)
            band_res = (field_res[0], b - a, field_res[2])
            ext = fa.band_halo_extract(wb, band_res, field_res, WS, shift)
            if s:
                want = L.band_halo_extract(ref, band_res, field_res, WS, shift)
                assert torch.equal(ext.cpu().float(), torch.from_numpy(np.ascontiguousarray(want)))
            else:
                assert ext is None
            backs[(r + 1) % world] = ext
        for r, (a, b) in enumerate(bands):
            band_res = (field_res[0], b - a, field_res[2])
            wb = torch.from_numpy(L.band_windows_of_field(wf.cpu().float().numpy(), field_res, WS, shift, a, b))
            wb = wb.to(dt_out).cuda()
            y = fa.crop_roll_unmerge_windows_band(wb, backs[r], band_res, field_res, WS, shift)
            assert torch.equal(y.cpu().float(), x[:, :, a:b].to(dt_out).cpu().float()), (world, r)


@pytest.mark.parametrize("shift", [(0, 0, 0), SHIFT])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_band_unmerge_adaln_bit_exact(shift, wdt):
    field_res, D = (4, 36, 72), 128
    C, H, W = field_res
    g = torch.Generator().manual_seed(3)
    _, _, _, _, nW, N = fa.util.window_geometry(field_res, WS, shift)
    win = torch.randn(nW, N, D, generator=g).to(wdt).cuda()
    resid = torch.randn(1, C * H * W, D, generator=g).cuda()
    scale = (torch.randn(1, 1, D, generator=g) * 0.1).cuda()
    shf = (torch.randn(1, 1, D, generator=g) * 0.1).cuda()
    full_bf = torch.empty(1, C * H * W, D, dtype=torch.bfloat16, device="cuda")
    full = fa.unmerge_adaptive_layernorm_film_add_residual(win, resid, scale, shf, field_res, WS, shift,
                                                           out_bf16=full_bf)
    full5 = full.view(1, C, H, W, D)
    full_bf5 = full_bf.view(1, C, H, W, D)
    resid5 = resid.view(1, C, H, W, D)
    _, ss = L.maybe_adjust_windows(WS, shift, field_res)
    s = ss[1]
    for world in (1, 2, 6):
        bands = sharding.band_bounds(field_res, WS, world)
        wbs = [torch.from_numpy(L.band_windows_of_field(win.cpu().float().numpy(), field_res, WS, shift, a, b))
               .to(wdt).cuda() for a, b in bands]
        for r, (a, b) in enumerate(bands):
            band_res = (C, b - a, W)
            pa, pb = bands[(r - 1) % world]
            halo_in = fa.band_halo_extract(wbs[(r - 1) % world], (C, pb - pa, W), field_res, WS, shift)
            res_b = resid5[:, :, a:b].reshape(1, -1, D).contiguous()
            ob = torch.empty(1, C * (b - a) * W, D, dtype=torch.bfloat16, device="cuda")
            y = fa.unmerge_adaptive_layernorm_film_add_residual_band(
                wbs[r], halo_in, res_b, scale, shf, band_res, field_res, WS, shift, out_bf16=ob)
            assert torch.equal(y.view(1, C, b - a, W, D), full5[:, :, a:b]), (world, r)
            assert torch.equal(ob.view(1, C, b - a, W, D), full_bf5[:, :, a:b])
            # The same rows in two launches: the rows past the halo depth first, without the
            # halo (as while it is in flight), then the first s rows.
            y2 = torch.full_like(y, float("nan"))
            ob2 = torch.full_like(ob, float("nan"))
            fa.unmerge_adaptive_layernorm_film_add_residual_band(
                wbs[r], None, res_b, scale, shf, band_res, field_res, WS, shift, out_bf16=ob2, out=y2,
                rows=(s, b - a - s))
            fa.unmerge_adaptive_layernorm_film_add_residual_band(
                wbs[r], halo_in, res_b, scale, shf, band_res, field_res, WS, shift, out_bf16=ob2, out=y2,
                rows=(0, s))
            assert torch.equal(y2, y) and torch.equal(ob2, ob), (world, r)
        if s == 0:
            break


@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_adaln_rows_split_equals_full(xdt):
    """Two row-range launches (the first s rows of every C slab, then the rest) write exactly what
    one full AdaLN + residual launch writes."""
    res, D = (4, 36, 72), 256
    C, H, W = res
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, C * H * W, D, generator=g).to(xdt).cuda()
    resid = torch.randn(2, C * H * W, D, generator=g).cuda()
    scale = (torch.randn(2, 1, D, generator=g) * 0.1).cuda()
    shf = (torch.randn(2, 1, D, generator=g) * 0.1).cuda()
    full_bf = torch.empty(2, C * H * W, D, dtype=torch.bfloat16, device="cuda")
    full = fa.adaptive_layernorm_film_add_residual_forward(resid, x, scale, shf, 0.0, 1e-5, output_fp32=True,
                                                           out_bf16=full_bf)
    out = torch.full_like(full, float("nan"))
    out_bf = torch.full_like(full_bf, float("nan"))
    fa.adaptive_layernorm_film_add_residual_rows(resid, x, scale, shf, res, (0, 3), 0.0, 1e-5, out=out,
                                                 out_bf16=out_bf)
    part = out.view(2, C, H, W, D)
    assert torch.isnan(part[:, :, 3:]).all() and not torch.isnan(part[:, :, :3]).any()
    fa.adaptive_layernorm_film_add_residual_rows(resid, x, scale, shf, res, (3, H - 3), 0.0, 1e-5, out=out,
                                                 out_bf16=out_bf)
    assert torch.equal(out, full) and torch.equal(out_bf, full_bf)


def test_band_rejects_bad_geometry():
    x = _x((4, 36, 72), 64, torch.float32)
    with pytest.raises(ValueError):  # band not a whole number of window rows
        fa.roll_pad_partition_windows_band(x[:, :, :9].contiguous(), x[:, :, 9:12].contiguous(), (4, 36, 72),
                                           WS, SHIFT)
    with pytest.raises(ValueError):  # missing halo on a shifted band
        fa.roll_pad_partition_windows_band(x[:, :, :12].contiguous(), None, (4, 36, 72), WS, SHIFT)
    with pytest.raises(ValueError):  # field height not a multiple of the window height
        y = _x((4, 45, 90), 64, torch.float32)
        fa.roll_pad_partition_windows_band(y[:, :, :6].contiguous(), y[:, :, 6:9].contiguous(), (4, 45, 90),
                                           WS, SHIFT)


def _stage(dim, heads, depth, precision, seed=5):
    torch.manual_seed(seed)
    layer = BasicLayer3D(dim=dim, depth=depth, num_heads=heads, ws=WS, time_dim=dim, precision=precision)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02)
    return layer.cuda().eval()


@pytest.mark.parametrize("precision,tol", [("fp32", 1e-6), ("bf16_mixed", 5e-3)])
@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("overlap", [False, True])
def test_sharded_stage_threads_match_field(precision, tol, world, overlap):
    field_res, dim, heads = (4, 36, 72), 128, 2
    C, H, W = field_res
    layer = _stage(dim, heads, 2, precision)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(1, C * H * W, dim, generator=g).cuda()
    c = torch.randn(1, dim, generator=g).cuda()
    with torch.no_grad():
        want, _ = layer(x, c, field_res)
    want5 = want.view(1, C, H, W, dim)
    x5 = x.view(1, C, H, W, dim)

    def fn(rank, ring):
        ctx = sharding.BandContext(field_res, WS, rank, world, ring=ring, timeout_s=60, overlap=overlap)
        a, b = ctx.h_begin, ctx.h_end
        xb = x5[:, :, a:b].reshape(1, -1, dim).contiguous()
        with torch.no_grad():
            yb, _ = layer(xb, c, ctx.res, band=ctx)
        torch.cuda.synchronize()
        return a, b, yb

    outs = sharding.run_ranks(world, fn, timeout_s=120)
    got = torch.cat([yb.view(1, C, b - a, W, dim) for a, b, yb in outs], dim=2)
    assert OB.relative_l2(got.cpu(), want5.cpu()) <= tol


# ------------------------------------------------------------------------ NCCL, one GPU per rank


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q, precision="fp32", overlap=False):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from flash_aurora_b200 import sharding as sh

        field_res, dim = (4, 36, 72), 128
        C, H, W = field_res
        layer = _stage(dim, 2, 2, precision)
        g = torch.Generator().manual_seed(9)
        x = torch.randn(1, C * H * W, dim, generator=g).cuda()
        c = torch.randn(1, dim, generator=g).cuda()
        group = sh.halo_process_group(timeout_s=60) if overlap else None
        ctx = sh.BandContext(field_res, WS, rank, world, group=group, timeout_s=60, overlap=overlap)
        a, b = ctx.h_begin, ctx.h_end
        with torch.no_grad():
            want, _ = layer(x, c, field_res)
            yb, _ = layer(x.view(1, C, H, W, dim)[:, :, a:b].reshape(1, -1, dim).contiguous(), c, ctx.res, band=ctx)
        want_b = want.view(1, C, H, W, dim)[:, :, a:b].reshape(1, -1, dim)
        err = OB.relative_l2(yb.cpu(), want_b.cpu())
        dist.barrier()
        q.put((rank, float(err)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("precision,tol", [("fp32", 1e-6), ("bf16_mixed", 5e-3)])
@pytest.mark.parametrize("overlap", [False, True])
def test_sharded_stage_nccl_two_gpus(precision, tol, overlap):
    """Two ranks over NCCL (NVLS off): each band of the sharded stage against the same rows of the
    unsharded stage, with the exchanges in line or on the side stream (high-priority halo group).
    In bf16_mixed the forward halo travels in bf16; cuBLAS may pick another algorithm for the
    band's row count, hence the bf16 tolerance."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q, precision, overlap)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, err = q.get(timeout=300)
        out[r] = err
    for p in procs:
        p.join(timeout=60)
    assert sorted(out) == [0, 1]
    assert all(e <= tol for e in out.values()), out
