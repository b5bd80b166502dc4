"""Device-side failures reach the host: a bounded wait that gives up inside a kernel is recorded in
a device status word and :func:`flash_aurora_b200.check_device_status` raises on it.

The failure is made without faulting anything: ``watchdog_selftest`` launches one warp that waits,
with a 1 ms limit, on an mbarrier nothing arrives on (the allowed way to make a wait run out on
this pool). After a reset a clean attention launch leaves the words at 0."""

from __future__ import annotations

import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200 import _lib
from flash_aurora_b200.pipeline import HostPipeline

pytestmark = pytest.mark.gpu


def _clean_attention():
    g = torch.Generator().manual_seed(1)
    qkv = (torch.randn(6, 144, 3 * 2 * 64, generator=g) * 0.1).bfloat16().cuda()
    return fa.window_attn_fwd_cute_qkvpacked(qkv, 2, output_layout="bnc")


def test_expired_wait_is_reported_then_cleared():
    fa.reset_device_status()
    assert fa.device_status() == {"attention": 0, "gemm": 0}
    fa.watchdog_selftest(timeout_ns=1_000_000)
    with pytest.raises(fa.DeviceStatusError) as ei:
        fa.check_device_status()
    assert ei.value.code == _lib.FA_STATUS_WATCHDOG_SELFTEST and ei.value.kernel == "attention"
    # check_device_status cleared the word; a clean launch keeps it at 0 and the context works.
    _clean_attention()
    fa.check_device_status()
    assert fa.device_status() == {"attention": 0, "gemm": 0}


def test_host_pipeline_wait_raises_on_device_failure():
    fa.reset_device_status()
    dev = torch.device("cuda", 0)

    def step(x):
        fa.watchdog_selftest(timeout_ns=200_000)
        return x * 2.0

    xs = [torch.randn(4, 8).pin_memory() for _ in range(2)]
    outs = [torch.empty(4, 8).pin_memory() for _ in range(2)]
    pipe = HostPipeline(step, dev)
    pipe.run(xs, outs)
    with pytest.raises(fa.DeviceStatusError):
        pipe.wait()
    for x, y in zip(xs, outs):  # the step's own results still arrived
        assert torch.equal(y, x * 2.0)
    fa.check_device_status()  # cleared by the raising check


def test_selftest_rejects_out_of_range_limits():
    with pytest.raises(ValueError, match="timeout_ns"):
        fa.watchdog_selftest(timeout_ns=10)
    with pytest.raises(ValueError, match="timeout_ns"):
        fa.watchdog_selftest(timeout_ns=10**9)
