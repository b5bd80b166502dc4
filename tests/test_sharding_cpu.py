"""Latitude-band sharding on CPU: band split, halo exchange over gloo ranks, fault injection.

The exchange code of ``flash_aurora_b200.sharding`` is backend-agnostic; here it moves CPU
tensors between gloo processes (world 2 and 4) and between thread-emulated ranks, and the band
windows are formed by the numpy oracle. Every band's windows must equal the matching rows of the
single-process partition of the whole field, bit for bit, and the halo-back round trip must
restore every band's tokens exactly.
"""

from __future__ import annotations

import os
import socket
import sys
import time

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import layout as L  # noqa: E402
from flash_aurora_b200 import sharding  # noqa: E402

WS = (2, 6, 12)
SHIFT = (1, 3, 6)


def test_band_bounds_split_window_rows():
    assert sharding.band_bounds((4, 360, 720), WS, 1) == [(0, 360)]
    b8 = sharding.band_bounds((4, 360, 720), WS, 8)
    assert b8[0] == (0, 42) and b8[-1] == (312, 360)
    assert all(e - s in (42, 48) for s, e in b8)
    assert all(b8[i][1] == b8[i + 1][0] for i in range(7))
    for world in (1, 2, 3, 4, 5, 8):
        assert sharding.band_bounds((4, 36, 72), WS, min(world, 6)) == L.band_split((4, 36, 72), WS, min(world, 6))
    with pytest.raises(ValueError):
        sharding.band_bounds((4, 45, 90), WS, 2)  # H not a multiple of the window height
    with pytest.raises(ValueError):
        sharding.band_bounds((4, 12, 24), WS, 3)  # fewer window rows than ranks


def _field(seed, field_res, D=8, B=1):
    g = np.random.default_rng(seed)
    return g.standard_normal((B,) + tuple(field_res) + (D,)).astype(np.float32)


def _rank_body(rank, world, ctx, x, field_res, shift):
    """One rank: forward halo, band windows vs field windows, halo-back, round trip."""
    a, b = ctx.h_begin, ctx.h_end
    _, ss = L.maybe_adjust_windows(WS, shift, field_res)
    s = ss[1]
    xb = torch.from_numpy(np.ascontiguousarray(x[:, :, a:b]))
    halo = ctx.halo_forward(xb, s).numpy() if s else None
    wb = L.band_partition(xb.numpy(), halo, field_res, WS, shift)
    wf = L.roll_pad_partition(x, field_res, WS, shift)
    ok_part = np.array_equal(wb, L.band_windows_of_field(wf, field_res, WS, shift, a, b))
    band_res = (field_res[0], b - a, field_res[2])
    halo_in = None
    if s:
        rows = torch.from_numpy(np.ascontiguousarray(L.band_halo_extract(wb, band_res, field_res, WS, shift)))
        halo_in = ctx.halo_back(rows).numpy()
    y = L.band_unmerge(wb, halo_in, band_res, field_res, WS, shift)
    ok_trip = np.array_equal(y, x[:, :, a:b])
    return ok_part, ok_trip


@pytest.mark.parametrize("world", [1, 2, 3, 6])
@pytest.mark.parametrize("shift", [(0, 0, 0), SHIFT])
def test_thread_ranks_match_field(world, shift):
    field_res = (4, 36, 72)
    x = _field(1, field_res)

    def fn(rank, ring):
        ctx = sharding.BandContext(field_res, WS, rank, world, ring=ring if world > 1 else None, timeout_s=30)
        return _rank_body(rank, world, ctx, x, field_res, shift)

    for ok_part, ok_trip in sharding.run_ranks(world, fn):
        assert ok_part and ok_trip


def test_thread_rank_failure_surfaces():
    """A rank that raises before its exchange: the others get HaloExchangeError, the caller the
    original error, and nothing hangs."""
    field_res = (4, 36, 72)
    x = _field(2, field_res)

    def fn(rank, ring):
        if rank == 1:
            raise KeyError("rank 1 failed before its halo exchange")
        ctx = sharding.BandContext(field_res, WS, rank, 3, ring=ring, timeout_s=30)
        return _rank_body(rank, 3, ctx, x, field_res, SHIFT)

    t0 = time.time()
    with pytest.raises((KeyError, sharding.HaloExchangeError)):
        sharding.run_ranks(3, fn, timeout_s=30)
    assert time.time() - t0 < 30


# ------------------------------------------------------------------------ gloo process ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, field_res, shift, mode, results):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from flash_aurora_b200 import sharding as sh

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        ctx = sh.BandContext(field_res, WS, rank, world, timeout_s=3.0)
        x = _field(5, field_res)
        if mode == "ok":
            results.put((rank, "ok", _rank_body(rank, world, ctx, x, field_res, shift)))
        elif mode == "silent_peer":
            # Rank 1 never sends: rank 0's receive must end in HaloExchangeError, not a hang.
            a, b = ctx.h_begin, ctx.h_end
            xb = torch.from_numpy(np.ascontiguousarray(x[:, :, a:b]))
            if rank == 0:
                t0 = time.time()
                try:
                    ctx.halo_forward(xb, 3)
                    results.put((rank, "no_error", time.time() - t0))
                except sh.HaloExchangeError as e:
                    results.put((rank, "timeout", (time.time() - t0, str(e)[:200])))
            else:
                # Post only the receive of rank 0's rows, never the send.
                recv = torch.empty_like(xb[:, :, :3])
                dist.irecv(recv, src=0).wait()
                time.sleep(6.0)
                results.put((rank, "silent", None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(world, field_res, shift, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, field_res, shift, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 120
    while len(out) < world and time.time() < deadline:
        try:
            r, kind, val = q.get(timeout=max(0.1, deadline - time.time()))
            out[r] = (kind, val)
        except Exception:
            break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,field_res", [(2, (4, 36, 72)), (4, (4, 36, 72)), (8, (4, 60, 24))])
def test_gloo_ranks_match_field(world, field_res):
    # world 8 over 10 window rows: bands of 1 or 2 window rows, uneven like config 5 at 8 GPUs
    out = _spawn(world, field_res, SHIFT, "ok")
    assert sorted(out) == list(range(world)), out
    for r, (kind, (ok_part, ok_trip)) in out.items():
        assert kind == "ok" and ok_part and ok_trip, (r, ok_part, ok_trip)


def test_gloo_silent_peer_times_out():
    out = _spawn(2, (4, 36, 72), SHIFT, "silent_peer")
    assert 0 in out, out
    kind, val = out[0]
    assert kind == "timeout", out
    elapsed, msg = val
    assert elapsed < 15 and "rank 0" in msg


@pytest.mark.parametrize("world", [2, 3])
def test_prefetched_forward_halo(world):
    """A forward halo issued early by the producing block (``prefetch_forward_halo``) is the one
    the shifted block's ``halo_forward`` returns: the next band's first rows. A prefetch issued for
    another tensor is refused, not silently used."""
    field_res = (4, 36, 72)
    x = _field(2, field_res)

    def fn(rank, ring):
        ctx = sharding.BandContext(field_res, WS, rank, world, ring=ring, timeout_s=30)
        xb = torch.from_numpy(np.ascontiguousarray(x[:, :, ctx.h_begin:ctx.h_end]))
        direct = ctx.halo_forward(xb, 3).clone()
        handle = ctx.prefetch_forward_halo(xb, 3)
        got = ctx.halo_forward(xb, 3).clone()
        nb = ctx.bounds[ctx.next][0]
        ok = torch.equal(direct, got) and np.array_equal(got.numpy(), x[:, :, nb:nb + 3])
        ok = ok and handle.recv.data_ptr() == ctx.buffer("fwd_recv", tuple(got.shape), got.dtype, "cpu").data_ptr()
        ctx.prefetch_forward_halo(xb, 3)
        try:
            ctx.halo_forward(xb.clone(), 3)
            refused = False
        except RuntimeError:
            refused = True
        return ok, refused

    for ok, refused in sharding.run_ranks(world, fn):
        assert ok and refused


def test_nccl_exchange_deadline_bookkeeping(monkeypatch):
    """The stream-ordered (NCCL) exchanges leave events that later exchanges and ``wait`` check:
    finished ones are dropped, and the oldest unfinished one past ``timeout_s`` raises
    HaloExchangeError after aborting the group (faked here: no GPU and no process group)."""
    import time

    from flash_aurora_b200.sharding import BandContext, HaloExchangeError

    class Ev:
        def __init__(self, done):
            self.done = done

        def query(self):
            return self.done

    ctx = BandContext((4, 36, 72), (2, 6, 12), 0, 2, timeout_s=5.0)
    aborted = []
    monkeypatch.setattr(ctx, "_abort", lambda: aborted.append(True))
    now = time.monotonic()
    ctx._pending = [(Ev(True), now - 100, 1, 1), (Ev(False), now, 1, 1)]
    ctx._check_pending(block=False)  # the finished one goes, the young unfinished one stays
    assert len(ctx._pending) == 1 and not aborted
    ctx._pending = [(Ev(False), now - 10, 1, 1)]
    with pytest.raises(HaloExchangeError, match="did not complete"):
        ctx.wait()
    assert aborted and ctx._pending == []
    ctx._pending = [(Ev(True), now, 1, 1)]
    ctx.wait()
    assert ctx._pending == []
