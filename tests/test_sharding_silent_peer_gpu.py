"""Failure detection of the NCCL halo exchange, on two GPUs, without faulting anything.

Both ranks make one halo exchange together; then rank 1 leaves the exchanges (between steps, with
nothing in flight: it only waits on the host) and rank 0 makes another. Rank 0's exchange has a
3 s host-side deadline: it must end in ``HaloExchangeError`` (the band context aborts the process
group, which ends NCCL's waiting transfer kernel), and rank 0's device must still run work
afterwards. NVLS is off (``NCCL_NVLS_ENABLE=0``); no kernel of this library waits on a peer.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import datetime
    import time

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from flash_aurora_b200.sharding import BandContext, HaloExchangeError

    store = dist.distributed_c10d._get_default_store()
    field_res = (4, 36, 72)
    ctx = BandContext(field_res, (2, 6, 12), rank, 2, timeout_s=3.0)
    xb = torch.randn(1, 4, ctx.h_end - ctx.h_begin, 72, 64, device="cuda")
    result = "?"
    try:
        ctx.halo_forward(xb, 3)  # both ranks: completes
        ctx.wait()
        dist.barrier()
        if rank == 1:
            result = "left"  # no further exchange; wait on the host for rank 0's verdict
            store.wait(["rank0_done"], datetime.timedelta(seconds=90))
        else:
            t0 = time.monotonic()
            try:
                ctx.halo_forward(xb, 3)
                ctx.wait()
                result = "no error"
            except HaloExchangeError:
                elapsed = time.monotonic() - t0
                # The device still runs work after the abort (on a fresh stream: the compute
                # stream was made to wait for the abandoned transfer).
                with torch.cuda.stream(torch.cuda.Stream()):
                    y = (torch.ones(1024, device="cuda") * 2).sum().item()
                result = f"raised after {elapsed:.1f} s, device ok ({y == 2048.0})"
            store.set("rank0_done", "1")
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result = f"unexpected {type(e).__name__}: {e}"
    q.put((rank, result))
    q.close()
    q.join_thread()
    os._exit(0)  # skip process-group teardown after an abort


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_silent_peer_raises_halo_exchange_error():
    import torch.multiprocessing as mp

    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, res = q.get(timeout=240)
        out[r] = res
    for p in procs:
        p.join(timeout=60)
    assert out[1] == "left", out
    assert out[0].startswith("raised") and out[0].endswith("(True)"), out
    secs = float(out[0].split()[2])
    assert 2.5 <= secs <= 30.0, out
