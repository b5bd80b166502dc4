"""Latitude-band sharding of a Swin3D field across ranks (one process per GPU).

The upstream backbone runs one field per device; its only multi-device path places whole
stages on different GPUs (engine/distributed/rollout_pipeline.py:137-169) and never splits a
field. Here a field ``(C, H, W)`` is split along H into bands of whole window rows, one band per
rank:

* windows are independent given their tokens and MLP/AdaLN are per token, so an unshifted block
  is fully local;
* a shifted block (H shift ``s = ws_h // 2``, swin3d.py:999-1001) rolls the field by ``-s`` rows
  (swin3d.py:757-770): the band's shifted windows start ``s`` rows into the band and end ``s``
  rows into the next band. Each rank therefore receives the next band's first ``s`` rows (the
  forward halo) before the partition, and after the attention it sends the outputs of its last
  ``s`` shifted rows back to their owner (the halo-back rows), which reads them in the fused
  unmerge + AdaLN. The last band wraps to band 0, exactly like ``torch.roll``.

Those two NCCL point-to-point exchanges per shifted block are the only collectives; there is no
remote TMA and no multicast. The shifted-window mask depends on the global window position, so a
band's region ids are the rows ``[h1_begin, h1_end)`` of the field's ``(nW, N)`` ids.

``exchange`` works for any backend: NCCL tensors on the GPU (the product path) and gloo CPU
tensors (the multi-process tests). Waits are bounded by ``timeout_s``: a peer that never sends
surfaces as :class:`HaloExchangeError` on the host, never as a hang. On NCCL the host does not
block per exchange (the transfers are stream-ordered); each exchange leaves a CUDA event, and
every later exchange, and :meth:`BandContext.wait`, checks the oldest unfinished one against the
deadline. On expiry the process group is aborted (which ends NCCL's spinning transfer kernels) and
:class:`HaloExchangeError` is raised.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from datetime import timedelta
from typing import Callable, Optional

import torch

from .util import maybe_adjust_windows

__all__ = [
    "HaloExchangeError",
    "HaloHandle",
    "halo_process_group",
    "band_bounds",
    "BandContext",
    "LocalRing",
]


class HaloExchangeError(RuntimeError):
    """A halo exchange with a neighbouring band did not complete."""


def halo_process_group(timeout_s: float = 60.0):
    """A NCCL process group over all ranks for the halo exchanges, whose internal streams have
    high priority: an exchange issued while a large kernel occupies the GPU gets its SMs as soon
    as blocks of that kernel retire, instead of after the whole kernel. A collective call: every
    rank calls it once, in the same order relative to its other group creations."""
    import torch.distributed as dist

    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    return dist.new_group(ranks=list(range(dist.get_world_size())), backend="nccl", pg_options=opts,
                          timeout=timedelta(seconds=timeout_s))


def band_bounds(field_res, window_size, world: int) -> list[tuple[int, int]]:
    """Token-row range ``[h_begin, h_end)`` of each rank's band.

    The field's window rows ``H // wh`` are split as evenly as possible (the first bands get the
    smaller share), so bands differ by at most one window row. Requires ``H % wh == 0`` and at
    least one window row per rank.
    """
    C, H, W = (int(v) for v in field_res)
    ws, _ = maybe_adjust_windows(tuple(window_size), (0, 0, 0), (C, H, W))
    wh = ws[1]
    if H % wh != 0:
        raise ValueError(f"band sharding needs H ({H}) to be a multiple of the window height ({wh})")
    rows = H // wh
    if world < 1 or world > rows:
        raise ValueError(f"cannot split {rows} window rows across {world} ranks")
    cuts = [(r * rows) // world for r in range(world + 1)]
    return [(cuts[r] * wh, cuts[r + 1] * wh) for r in range(world)]


@dataclass
class LocalRing:
    """In-process stand-in for the ranks of a ring: ``world`` threads of one process exchange
    tensors through shared slots. Used to run several bands on one device (tests, and the
    single-process check of the sharded block); every participant must call ``exchange`` the
    same number of times, as with a real process group."""

    world: int
    timeout_s: float = 60.0
    _slots: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        import threading

        self._barrier = threading.Barrier(self.world, timeout=self.timeout_s)

    def exchange(self, rank: int, send: torch.Tensor, recv: torch.Tensor, dst: int, src: int) -> None:
        import threading

        try:
            self._slots[(rank, dst)] = send
            self._barrier.wait()
            recv.copy_(self._slots[(src, rank)])
            self._barrier.wait()
        except threading.BrokenBarrierError as e:
            raise HaloExchangeError(f"rank {rank}: local ring exchange with rank {src} timed out") from e
        finally:
            self._slots.pop((rank, dst), None)


class BandContext:
    """One rank's band of a field plus the halo exchanges with its neighbours.

    ``group``: a ``torch.distributed`` process group (default: the world group) when the ranks
    are processes; ``ring``: a :class:`LocalRing` when they are threads of one process; neither
    when ``world == 1`` (the band is the whole field and the halo wraps onto itself).
    """

    def __init__(self, field_res, window_size, rank: int, world: int, *, group=None,
                 ring: Optional[LocalRing] = None, timeout_s: float = 60.0,
                 overlap: Optional[bool] = None) -> None:
        self.field_res = tuple(int(v) for v in field_res)
        self.window_size = tuple(int(v) for v in window_size)
        self.rank, self.world = int(rank), int(world)
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.bounds = band_bounds(self.field_res, self.window_size, self.world)
        self.h_begin, self.h_end = self.bounds[self.rank]
        self.group = group
        self.ring = ring
        self.timeout_s = float(timeout_s)
        # Overlap the halo exchanges with the rows that do not need them. Default: from four
        # ranks on (FA_BAND_OVERLAP=0 / 1 or overlap=False / True override it). Measured on the
        # config-5 stage: on two B200s 0.4-0.7 ms per 52 ms step slower with it (the two extra
        # short launches per exchange cost more than the exchange they hide), on four 0.35-0.4 ms
        # per 25 ms step faster (smaller bands, the same exchanges).
        if overlap is None:
            env = os.environ.get("FA_BAND_OVERLAP")
            overlap = (env == "1") if env in ("0", "1") else self.world >= 4
        self.overlap = bool(overlap)
        self.prev = (self.rank - 1) % self.world
        self.next = (self.rank + 1) % self.world
        self._gids: dict = {}
        self._bufs: dict = {}
        # Unfinished NCCL exchanges: (event after the transfers, host time issued, dst, src).
        self._pending: list = []
        self._streams: dict = {}
        # Forward halo issued by the previous block for the next shifted block: (key, handle).
        self._fwd_prefetch = None

    # ------------------------------------------------------------------ geometry
    @property
    def res(self) -> tuple[int, int, int]:
        """The band's own resolution ``(C, H_band, W)``."""
        C, _, W = self.field_res
        return (C, self.h_end - self.h_begin, W)

    def window_rows(self, window_size) -> tuple[int, int]:
        ws, _ = maybe_adjust_windows(tuple(window_size), (0, 0, 0), self.field_res)
        return self.h_begin // ws[1], self.h_end // ws[1]

    def group_ids(self, window_size, shift_size, warped: bool, device) -> Optional[torch.Tensor]:
        """The band's ``(nW_band, N)`` region ids, or ``None`` for an unshifted block."""
        from .window_attn import mark_region_ids_fit, shifted_window_group_ids

        ws, ss = maybe_adjust_windows(tuple(window_size), tuple(shift_size), self.field_res)
        if not any(ss):
            return None
        key = (ws, ss, bool(warped), str(device))
        hit = self._gids.get(key)
        if hit is None:
            full = shifted_window_group_ids(self.field_res, tuple(window_size), tuple(shift_size), warped, device)
            C, H, W = self.field_res
            g1 = [-(-d // w) for d, w in zip((C, H, W), ws)]
            a, b = self.h_begin // ws[1], self.h_end // ws[1]
            hit = full.view(g1[0], g1[1], g1[2], -1)[:, a:b].reshape(-1, full.shape[-1]).contiguous()
            # The band's windows are a subset of the field's: the field's tensor-core fit carries over.
            mark_region_ids_fit(hit, getattr(full, "_fa_regions_fit", False))
            self._gids[key] = hit
        return hit

    # ------------------------------------------------------------------ exchanges
    def buffer(self, name: str, shape, dtype, device) -> torch.Tensor:
        """Persistent receive/send buffer, reused across calls of the same shape."""
        key = (name, tuple(shape), dtype, str(device))
        buf = self._bufs.get(key)
        if buf is None:
            buf = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[key] = buf
        return buf

    def exchange(self, send: torch.Tensor, recv: torch.Tensor, dst: int, src: int) -> None:
        """Send ``send`` to rank ``dst`` and receive ``recv`` from rank ``src``.

        NCCL: both transfers are queued on NCCL's stream ordered after the current stream's work,
        and the current stream waits for them; the host does not block. gloo: the host waits at
        most ``timeout_s``. Failures raise :class:`HaloExchangeError`.
        """
        if self.world == 1:
            recv.copy_(send)
            return
        if self.ring is not None:
            self.ring.exchange(self.rank, send, recv, dst, src)
            return
        import torch.distributed as dist

        try:
            g = self.group
            gdst = dst if g is None else dist.get_global_rank(g, dst)
            gsrc = src if g is None else dist.get_global_rank(g, src)
            works = dist.batch_isend_irecv([
                dist.P2POp(dist.isend, send.contiguous(), gdst, g),
                dist.P2POp(dist.irecv, recv, gsrc, g),
            ])
            cuda = recv.is_cuda
            for w in works:
                if cuda:
                    w.wait()  # the current stream waits; the host does not
                else:
                    w.wait(timedelta(seconds=self.timeout_s))
            if cuda:
                ev = torch.cuda.Event()
                ev.record()
                self._pending.append((ev, time.monotonic(), dst, src))
                self._check_pending(block=False)
        except HaloExchangeError:
            raise
        except RuntimeError as e:
            raise HaloExchangeError(
                f"rank {self.rank}: halo exchange (send to {dst}, receive from {src}) failed: {e}") from e

    def _overlapped(self, t: torch.Tensor) -> bool:
        """Exchanges of ``t`` run on a side stream: NCCL between processes only (gloo and the
        thread ring exchange on the host, a single band copies locally)."""
        return t.is_cuda and self.world > 1 and self.ring is None

    def comm_stream(self, device) -> "torch.cuda.Stream":
        """The side stream that overlapped exchanges (and their staging copies) run on."""
        key = str(device)
        st = self._streams.get(key)
        if st is None:
            st = torch.cuda.Stream(device=device, priority=-1)  # high priority, like the NCCL streams
            self._streams[key] = st
        return st

    def exchange_async(self, send: torch.Tensor, recv: torch.Tensor, dst: int, src: int,
                       stage: Optional[Callable[[], None]] = None) -> "HaloHandle":
        """:meth:`exchange` ordered after the current stream's work so far but run on the side
        stream, so the current stream can go on with work that does not need ``recv``; the
        returned handle's :meth:`HaloHandle.wait` orders the current stream after the transfer.
        ``stage`` (optional) fills ``send`` first, on the side stream. Without a side stream
        (gloo, the thread ring, one band) the exchange completes before this returns."""
        if not self._overlapped(recv):
            if stage is not None:
                stage()
            self.exchange(send, recv, dst, src)
            return HaloHandle(recv, None)
        cur = torch.cuda.current_stream(recv.device)
        comm = self.comm_stream(recv.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        with torch.cuda.stream(comm):
            comm.wait_event(ready)
            if stage is not None:
                stage()
            self.exchange(send, recv, dst, src)
            done = torch.cuda.Event()
            done.record(comm)
        return HaloHandle(recv, done)

    def _check_pending(self, block: bool) -> None:
        """Drop finished exchanges; raise when the oldest unfinished one is past the deadline.
        With ``block`` poll until every pending exchange finished or the deadline passed."""
        while self._pending:
            ev, t0, dst, src = self._pending[0]
            if ev.query():
                self._pending.pop(0)
                continue
            if time.monotonic() - t0 > self.timeout_s:
                self._pending.clear()
                self._abort()
                raise HaloExchangeError(
                    f"rank {self.rank}: halo exchange (send to {dst}, receive from {src}) did not complete "
                    f"within {self.timeout_s:.0f} s")
            if not block:
                return
            time.sleep(0.001)

    def _abort(self) -> None:
        """End the group's communicator so that its transfer kernels stop waiting for the peer."""
        try:
            import torch.distributed as dist
            from torch.distributed import distributed_c10d as c10d

            abort = getattr(c10d, "_abort_process_group", None)
            if abort is not None and dist.is_initialized():
                abort(self.group if self.group is not None else dist.group.WORLD)
        except Exception:  # noqa: BLE001 - the exchange error is what the caller must see
            pass

    def wait(self) -> None:
        """Block until every exchange issued so far has completed on the device, or raise
        :class:`HaloExchangeError` once the oldest of them is ``timeout_s`` old."""
        self._check_pending(block=True)

    def halo_forward(self, x_band: torch.Tensor, s: int, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """Receive the next band's first ``s`` rows: ``x_band (B, C, Hb, W, D)`` -> ``(B, C, s, W, D)``.

        This rank sends its own first ``s`` rows to the previous band at the same time. When the
        block that produced ``x_band`` already issued that exchange (:meth:`prefetch_forward_halo`)
        the current stream only waits for it.
        """
        B, C, _, W, D = x_band.shape
        dtype = x_band.dtype if dtype is None else dtype
        key = (x_band.data_ptr(), tuple(x_band.shape), int(s), dtype)
        pre, self._fwd_prefetch = self._fwd_prefetch, None
        if pre is not None:
            if pre[0] != key:
                raise RuntimeError("the prefetched forward halo was issued for another tensor or shift")
            return pre[1].wait()
        return self.prefetch_forward_halo(x_band, s, dtype, _keep=False).wait()

    def prefetch_forward_halo(self, x_band: torch.Tensor, s: int, dtype: Optional[torch.dtype] = None, *,
                              _keep: bool = True) -> "HaloHandle":
        """Issue the forward-halo exchange of ``x_band`` now, as soon as its first ``s`` rows are
        written, so that it overlaps the rest of the producing block; the next shifted block's
        :meth:`halo_forward` of the same tensor waits for it. Every rank must prefetch for the same
        blocks (the exchanges pair up in issue order)."""
        B, C, _, W, D = x_band.shape
        dtype = x_band.dtype if dtype is None else dtype
        send = self.buffer("fwd_send", (B, C, s, W, D), dtype, x_band.device)
        recv = self.buffer("fwd_recv", (B, C, s, W, D), dtype, x_band.device)
        if self._overlapped(recv):
            # The side stream reads x_band: keep its memory from the allocator until it has.
            x_band.record_stream(self.comm_stream(x_band.device))
        handle = self.exchange_async(send, recv, dst=self.prev, src=self.next,
                                     stage=lambda: send.copy_(x_band[:, :, :s]))
        if _keep:
            self._fwd_prefetch = ((x_band.data_ptr(), tuple(x_band.shape), int(s), dtype), handle)
        return handle

    def halo_back(self, rows: torch.Tensor) -> torch.Tensor:
        """Send the halo-back rows ``(B, C, s, W, D)`` to the next band; receive this band's own
        first ``s`` rows, computed by the previous band."""
        return self.halo_back_async(rows).wait()

    def halo_back_async(self, rows: torch.Tensor) -> "HaloHandle":
        """:meth:`halo_back` on the side stream: the caller normalises the band rows that need
        no halo meanwhile and waits on the handle before the first ``s`` rows."""
        recv = self.buffer("back_recv", tuple(rows.shape), rows.dtype, rows.device)
        return self.exchange_async(rows, recv, dst=self.next, src=self.prev)


class HaloHandle:
    """A halo exchange in flight: :meth:`wait` orders the current stream after the transfer and
    returns the receive buffer."""

    def __init__(self, recv: torch.Tensor, done: Optional["torch.cuda.Event"]) -> None:
        self.recv = recv
        self.done = done

    def wait(self) -> torch.Tensor:
        if self.done is not None:
            torch.cuda.current_stream(self.recv.device).wait_event(self.done)
        return self.recv


def run_ranks(world: int, fn: Callable[[int, LocalRing], object], timeout_s: float = 120.0) -> list:
    """Run ``fn(rank, ring)`` for ``world`` emulated ranks on threads of this process and return
    their results in rank order; the first exception of any rank is re-raised."""
    import threading

    ring = LocalRing(world, timeout_s=timeout_s)
    out: list = [None] * world
    err: list = [None] * world

    def body(r: int) -> None:
        try:
            out[r] = fn(r, ring)
        except BaseException as e:  # noqa: BLE001 - re-raised in the caller
            err[r] = e
            ring._barrier.abort()

    ts = [threading.Thread(target=body, args=(r,), daemon=True) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout_s)
    for e in err:
        if e is not None:
            raise e
    if any(t.is_alive() for t in ts):
        raise HaloExchangeError(f"emulated ranks did not finish within {timeout_s} s")
    return out
