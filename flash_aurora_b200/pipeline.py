"""Host-resident inputs and outputs streamed through a device step with overlapped copies.

A forecast service feeds the backbone one field after another (ensemble members, or successive
rollout inputs) from pinned host memory and reads every result back. Run serially, each step
pays its host-to-device copy, the step, and its device-to-host copy one after another; the
copies use the copy engines, not the SMs, so they can run under the neighbouring steps.
:class:`HostPipeline` double-buffers the device input: step ``i + 1``'s upload runs on one copy
stream while step ``i`` computes, and step ``i``'s download runs on another copy stream while
step ``i + 1`` computes. Every step still moves its own input and output across PCIe; only the
waiting is removed. Ordering is by CUDA events only; the host never blocks inside ``run``.

The step is either a callable (the pipeline keeps ``depth`` device input buffers) or a sequence of
captured graphs (:func:`~flash_aurora_b200.graph.capture_slots`): then step ``i`` uploads straight
into slot ``i % len(slots)``'s static input, replays it and downloads its static output, so no
device-side copy enters or leaves the graphs; a slot is replayed again only after the download of
its previous output.
:meth:`HostPipeline.wait` is the sync point: it blocks until the last download has landed and
then checks the kernels' device status words (a pipeline wait that gave up inside a kernel is
reported there, not by the launch), raising :class:`~flash_aurora_b200.status.DeviceStatusError`.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch

__all__ = ["HostPipeline"]


def _download_half(host_out: torch.Tensor, src: torch.Tensor, right: bool, stream) -> None:
    """One strided device-to-host copy into the left or right half of the last dimension of the
    contiguous pinned ``host_out`` (rows of ``2 * D`` elements): from ``src`` rows of ``D`` elements
    (``right``), or from the left half of ``src`` rows of ``2 * D`` elements."""
    from cuda.bindings import runtime as rt

    if not host_out.is_contiguous() or host_out.device.type != "cpu":
        raise ValueError("host outputs must be contiguous host tensors")
    if src.stride(-1) != 1 or not (src.is_contiguous() or src.numel() == src.shape[-2] * src.shape[-1]):
        raise ValueError("the source must be a contiguous tensor of rows")
    e = host_out.element_size()
    d2 = host_out.shape[-1]
    rows = host_out.numel() // d2
    width = (d2 // 2) * e
    dst = host_out.data_ptr() + (width if right else 0)
    spitch = src.stride(-2) * e if src.dim() >= 2 else width
    err, = rt.cudaMemcpy2DAsync(dst, d2 * e, src.data_ptr(), spitch, width, rows,
                                rt.cudaMemcpyKind.cudaMemcpyDeviceToHost, stream.cuda_stream)
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaMemcpy2DAsync failed: {err}")


class HostPipeline:
    """``run(host_inputs, host_outputs)`` computes ``host_outputs[i] = step(host_inputs[i])``.

    ``step`` takes a device tensor shaped like the inputs and returns a device tensor shaped like
    the outputs; it runs on the caller's current stream. Inputs and outputs should be pinned
    host tensors (pageable memory works but serialises the copies).
    """

    def __init__(self, step, device, depth: int = 2) -> None:
        self.slots = None
        if isinstance(step, (list, tuple)):
            # Captured slots: objects with static_input, static_output and replay().
            if not step or not all(hasattr(t, "replay") and hasattr(t, "static_input") for t in step):
                raise ValueError("slots must be a non-empty sequence of captured steps")
            self.slots = list(step)
            depth = len(self.slots)
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.step = step
        self.device = torch.device(device)
        self.depth = depth
        self.up = torch.cuda.Stream(self.device)
        self.down = torch.cuda.Stream(self.device)
        self._bufs: list[torch.Tensor] = []
        self._last: torch.cuda.Event | None = None

    def _buffers(self, like: torch.Tensor) -> list[torch.Tensor]:
        if not self._bufs or self._bufs[0].shape != like.shape or self._bufs[0].dtype != like.dtype:
            self._bufs = [torch.empty(like.shape, dtype=like.dtype, device=self.device) for _ in range(self.depth)]
        return self._bufs

    def run(self, host_inputs: Sequence[torch.Tensor], host_outputs: Sequence[torch.Tensor]) -> None:
        if len(host_inputs) != len(host_outputs):
            raise ValueError("need one output tensor per input tensor")
        n = len(host_inputs)
        if n == 0:
            return
        if self.slots is not None:
            return self._run_slots(host_inputs, host_outputs)
        compute = torch.cuda.current_stream(self.device)
        bufs = self._buffers(host_inputs[0])
        uploaded = [torch.cuda.Event() for _ in range(n)]
        consumed = [torch.cuda.Event() for _ in range(n)]  # step i no longer reads its input buffer
        start = torch.cuda.Event()
        start.record(compute)
        self.up.wait_event(start)
        self.down.wait_event(start)

        def upload(i: int) -> None:
            with torch.cuda.stream(self.up):
                if i >= self.depth:
                    self.up.wait_event(consumed[i - self.depth])
                bufs[i % self.depth].copy_(host_inputs[i], non_blocking=True)
                uploaded[i].record(self.up)

        for i in range(min(self.depth - 1, n)):
            upload(i)
        last_down = None
        for i in range(n):
            if i + self.depth - 1 < n:
                upload(i + self.depth - 1)
            compute.wait_event(uploaded[i])
            y = self.step(bufs[i % self.depth])
            consumed[i].record(compute)
            done = torch.cuda.Event()
            done.record(compute)
            with torch.cuda.stream(self.down):
                self.down.wait_event(done)
                y.record_stream(self.down)
                host_outputs[i].copy_(y, non_blocking=True)
                last_down = torch.cuda.Event()
                last_down.record(self.down)
            del y
        # The caller's stream ends after the last download, so events recorded on it after
        # run() returns bracket all the copies.
        compute.wait_event(last_down)
        self._last = last_down

    def _run_slots(self, host_inputs, host_outputs) -> None:
        n, k = len(host_inputs), len(self.slots)
        compute = torch.cuda.current_stream(self.device)
        for t in self.slots:
            if tuple(t.static_input.shape) != tuple(host_inputs[0].shape):
                raise ValueError(f"slots captured for {tuple(t.static_input.shape)}, inputs are "
                                 f"{tuple(host_inputs[0].shape)}")
        uploaded = [torch.cuda.Event() for _ in range(n)]
        computed = [torch.cuda.Event() for _ in range(n)]    # replay i done: slot input and output free to reuse
        downloaded = [torch.cuda.Event() for _ in range(n)]  # output i in host memory
        start = torch.cuda.Event()
        start.record(compute)
        self.up.wait_event(start)
        self.down.wait_event(start)

        def upload(i: int) -> None:
            with torch.cuda.stream(self.up):
                if i >= k:
                    self.up.wait_event(computed[i - k])  # the slot's previous replay read its input
                self.slots[i % k].static_input.copy_(host_inputs[i], non_blocking=True)
                uploaded[i].record(self.up)

        for i in range(min(k - 1, n)):
            upload(i)
        for i in range(n):
            if i + k - 1 < n:
                upload(i + k - 1)
            slot = self.slots[i % k]
            compute.wait_event(uploaded[i])
            if i >= k:
                compute.wait_event(downloaded[i - k])  # the slot's previous output has left
            slot.replay()
            computed[i].record(compute)
            with torch.cuda.stream(self.down):
                if getattr(slot, "skip_ready", None) is not None:
                    # The skip half leaves as soon as the graph has written it, the decoder half
                    # after the replay (capture_backbone_slots).
                    self.down.wait_event(slot.skip_ready)
                    _download_half(host_outputs[i], slot.skip, right=True, stream=self.down)
                    self.down.wait_event(computed[i])
                    _download_half(host_outputs[i], slot.static_output, right=False, stream=self.down)
                else:
                    self.down.wait_event(computed[i])
                    host_outputs[i].copy_(slot.static_output, non_blocking=True)
                downloaded[i].record(self.down)
        compute.wait_event(downloaded[n - 1])
        self._last = downloaded[n - 1]

    def wait(self, check_status: bool = True) -> None:
        """Block until the outputs of the last :meth:`run` are in host memory; then, with
        ``check_status``, raise if a kernel recorded a device-side failure meanwhile."""
        if self._last is not None:
            self._last.synchronize()
        if check_status:
            from .status import check_device_status

            check_device_status(self.device)
