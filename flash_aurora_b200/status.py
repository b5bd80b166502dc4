"""Device-side failure status of the pipelined kernels, surfaced on the host.

The attention and GEMM kernels bound every wait of their producer/consumer pipelines. A wait that
gives up (a stuck pipeline), or a region-id tensor tagged as fitting the tensor-core mask that does
not fit (that window is then left unmasked), is recorded in a device status word instead of
hanging or faulting. The launch itself returns normally, so callers check the words at a point
where they synchronise anyway: after a batch of steps, after reading results back
(:meth:`flash_aurora_b200.pipeline.HostPipeline.wait` does), or after a graph replay.
:func:`check_device_status` raises :class:`DeviceStatusError` when either word is set.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

__all__ = ["DeviceStatusError", "device_status", "check_device_status", "reset_device_status",
           "watchdog_selftest"]

_MEANING = {
    _lib.FA_STATUS_REGIONS_BROKEN: "region ids tagged as fitting the tensor-core mask had more than 16 distinct "
                                   "ids (or an id >= 32) in a window; that window was computed unmasked",
    _lib.FA_STATUS_WATCHDOG_SELFTEST: "the watchdog self-test wait expired (expected after watchdog_selftest)",
}


class DeviceStatusError(RuntimeError):
    """A kernel of this library recorded a failure in its device status word."""

    def __init__(self, kernel: str, code: int) -> None:
        self.kernel, self.code = kernel, int(code)
        what = _MEANING.get(self.code, "a bounded pipeline wait gave up and the kernel returned early; "
                                       "its output is incomplete")
        super().__init__(f"{kernel} device status {self.code}: {what}")


def device_status(device: Optional[torch.device] = None) -> dict:
    """``{"attention": code, "gemm": code}`` of ``device`` (0 = clean). Synchronises the device."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        torch.cuda.synchronize(dev)
        out = {}
        for name, fn in (("attention", lib.fa_attention_status), ("gemm", lib.fa_gemm_status)):
            v = ctypes.c_int(0)
            _lib.check(fn(ctypes.byref(v)), f"fa_{name}_status")
            out[name] = int(v.value)
    return out


def reset_device_status(device: Optional[torch.device] = None) -> None:
    """Clear both status words (ordered on the current stream of ``device``)."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        s = _lib.stream_ptr(dev)
        _lib.check(lib.fa_attention_status_reset(s), "fa_attention_status_reset")
        _lib.check(lib.fa_gemm_status_reset(s), "fa_gemm_status_reset")


def check_device_status(device: Optional[torch.device] = None, reset: bool = True) -> None:
    """Raise :class:`DeviceStatusError` if a kernel recorded a failure since the last reset.
    With ``reset`` the words are cleared after they are read (also when raising)."""
    st = device_status(device)
    if reset and any(st.values()):
        reset_device_status(device)
    for name in ("attention", "gemm"):
        if st[name]:
            raise DeviceStatusError(name, st[name])


def watchdog_selftest(timeout_ns: int = 1_000_000, device: Optional[torch.device] = None) -> None:
    """Launch the bounded-wait self-test (``fa_watchdog_selftest``): a wait on an mbarrier that
    nothing arrives on gives up after ``timeout_ns`` and records its code; nothing faults."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().fa_watchdog_selftest(int(timeout_ns), _lib.stream_ptr(dev)), "watchdog_selftest")
