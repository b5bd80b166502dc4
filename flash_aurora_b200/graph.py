"""A static-shape step (the backbone forward) captured once into a CUDA graph and replayed.

A forecast service runs the backbone on inputs of one shape over and over. Its ~560 kernel
launches per step cost the host about 13 ms of launch work, which mostly hides behind the GPU's
~100 ms, but every short gap between kernels is GPU idle time. Replaying a captured graph removes
those gaps (about 2 % of the step here) and the per-step Python work.

The capture runs ``fn`` a few times on a side stream first, so that every cache the step fills
lazily (tensor-core weight copies, region ids, window buffers) exists before capture, then records
one call. The graph reads ``static_input`` and writes ``static_output``; both live as long as the
object.
"""

from __future__ import annotations

from typing import Callable

import torch

__all__ = ["CapturedStep", "capture_slots", "capture_backbone_slots"]


class CapturedStep:
    """``fn(x) -> y`` captured for inputs shaped like ``example`` (a CUDA tensor)."""

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], example: torch.Tensor, warmup: int = 2) -> None:
        if not example.is_cuda:
            raise ValueError("CapturedStep needs a CUDA example input")
        self.static_input = example.detach().clone()
        side = torch.cuda.Stream(example.device)
        side.wait_stream(torch.cuda.current_stream(example.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                fn(self.static_input)
        torch.cuda.current_stream(example.device).wait_stream(side)
        # keep_graph: the captured graph stays queryable (kernel_names) after instantiation.
        self.graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(self.graph):
            self.static_output = fn(self.static_input)
        self.graph.instantiate()

    def kernel_names(self) -> list[str]:
        """The (mangled) name of every kernel node of the captured graph: one entry per kernel
        launch of a replay, this library's and the libraries' (cuBLAS, PyTorch) alike. A name
        that cannot be resolved is returned as ``"?"``; the count stays exact."""
        from cuda.bindings import driver as cu
        from cuda.bindings import runtime as rt

        g = rt.cudaGraph_t(init_value=int(self.graph.raw_cuda_graph()))
        err, _, n = rt.cudaGraphGetNodes(g, 0)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaGraphGetNodes failed: {err}")
        err, nodes, n = rt.cudaGraphGetNodes(g, n)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaGraphGetNodes failed: {err}")
        names = []
        for node in nodes[:n]:
            err, kind = rt.cudaGraphNodeGetType(node)
            if err != rt.cudaError_t.cudaSuccess or kind != rt.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                continue
            name = "?"
            try:
                err, params = cu.cuGraphKernelNodeGetParams(cu.CUgraphNode(init_value=int(node)))
                if err == cu.CUresult.CUDA_SUCCESS:
                    err, raw = cu.cuFuncGetName(params.func)
                    if err == cu.CUresult.CUDA_SUCCESS and raw:
                        name = raw.decode() if isinstance(raw, bytes) else str(raw)
            except Exception:  # noqa: BLE001 - the count does not depend on the name
                pass
            names.append(name)
        return names

    def replay(self) -> torch.Tensor:
        """Run the step on the current contents of ``static_input``; returns ``static_output``
        (overwritten by the next replay)."""
        self.graph.replay()
        return self.static_output

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """Copy ``x`` into the static input, replay, and return a fresh copy of the output."""
        if x.shape != self.static_input.shape or x.dtype != self.static_input.dtype:
            raise ValueError(f"captured for {tuple(self.static_input.shape)} {self.static_input.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        self.static_input.copy_(x)
        self.graph.replay()
        return self.static_output.clone()


def capture_slots(fn: Callable[[torch.Tensor], torch.Tensor], example: torch.Tensor, n: int = 2,
                  warmup: int = 2) -> list[CapturedStep]:
    """``n`` captures of the same step, each with its own static input and output and its own
    memory pool, for :class:`~flash_aurora_b200.pipeline.HostPipeline`: while slot ``k``
    computes, the previous slot's output is still being downloaded and the next slot's input is
    being uploaded, with no device-side copy in or out of the graphs. (Two captures sharing one
    pool produced wrong outputs in this rotation, so each slot keeps its own intermediates.)"""
    if n < 1:
        raise ValueError("n must be >= 1")
    return [CapturedStep(fn, example, warmup=warmup if i == 0 else 0) for i in range(n)]


def capture_backbone_slots(model, lead_time, rollout_step: int, patch_res, example: torch.Tensor,
                           n: int = 2, warmup: int = 2) -> list[CapturedStep]:
    """:func:`capture_slots` for a :class:`~flash_aurora_b200.swin3d.Swin3DTransformerBackbone`
    forward whose output is ``cat([decoder output, skip], -1)``: each slot also carries ``skip``
    (its graph's first-encoder-layer output, the right half of that concatenation) and
    ``skip_ready``, an event recorded inside the graph right after ``skip`` is written, so that
    :class:`~flash_aurora_b200.pipeline.HostPipeline` downloads that half while the decoder still
    runs and only the left half after the replay."""
    if n < 1:
        raise ValueError("n must be >= 1")
    step = lambda x: model(x, lead_time=lead_time, rollout_step=rollout_step, patch_res=patch_res)
    slots = []
    try:
        for i in range(n):
            ev = torch.cuda.Event(external=True)
            seen: list = []

            def hook(t: torch.Tensor, ev=ev, seen=seen) -> None:
                ev.record()
                seen.append(t)

            model.skip_hook = hook
            slot = CapturedStep(step, example, warmup=warmup if i == 0 else 0)
            if not seen:
                raise ValueError("the model never called skip_hook (no encoder layer?)")
            slot.skip = seen[-1]  # the tensor the capture recorded (the graph rewrites it in place)
            slot.skip_ready = ev
            if (slot.static_output.dim() != 3 or slot.skip.shape[:2] != slot.static_output.shape[:2]
                    or 2 * slot.skip.shape[-1] != slot.static_output.shape[-1]):
                raise ValueError("the step's output is not cat([decoder output, skip], -1)")
            slots.append(slot)
    finally:
        model.skip_hook = None
    return slots
