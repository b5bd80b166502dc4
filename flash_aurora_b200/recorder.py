"""Optional per-launch timing of the block's operators, for the benchmark's step breakdown.

When a :class:`StepRecorder` is installed with :func:`set_step_recorder`, the block forward brackets
each of its operators (partition, QKV GEMM, attention, proj GEMM, the two AdaLN kernels, fc1 + GELU,
fc2) with CUDA events on the current stream and records the operator's algorithmic bytes and
FLOPs. Nothing is recorded, and nothing is synchronised, when no recorder is installed; a CUDA
graph is never captured with one installed (events cannot be timed inside a graph).
"""

from __future__ import annotations

from typing import Optional

import torch

__all__ = ["KernelRecorder", "StepRecorder", "set_step_recorder", "step_recorder", "begin", "end"]


class KernelRecorder:
    """Launches of one operator: ``records`` holds ``(event0, event1, bytes, flops)``."""

    def __init__(self) -> None:
        self.records: list[tuple[torch.cuda.Event, torch.cuda.Event, int, int]] = []

    def totals(self) -> tuple[float, int, int, int]:
        """(milliseconds, bytes, flops, launches) summed over the recorded launches."""
        ms = sum(a.elapsed_time(b) for a, b, _, _ in self.records)
        return ms, sum(r[2] for r in self.records), sum(r[3] for r in self.records), len(self.records)

    def by_shape(self) -> list[tuple[int, int, float]]:
        """(bytes per launch, launches, average milliseconds) per distinct launch size, largest
        first: the per-stage view of the same launches."""
        acc: dict[int, list[float]] = {}
        for a, b, nbytes, _ in self.records:
            acc.setdefault(nbytes, []).append(a.elapsed_time(b))
        return [(nb, len(v), sum(v) / len(v)) for nb, v in sorted(acc.items(), key=lambda kv: -kv[0])]


class StepRecorder:
    """One :class:`KernelRecorder` per operator name."""

    def __init__(self) -> None:
        self.kinds: dict[str, KernelRecorder] = {}

    def get(self, kind: str) -> KernelRecorder:
        rec = self.kinds.get(kind)
        if rec is None:
            rec = self.kinds[kind] = KernelRecorder()
        return rec

    def summary(self, steps: int) -> dict:
        """``{kind: {"ms_per_step", "bytes_per_step", "flops_per_step", "launches_per_step"}}``."""
        out = {}
        for kind, rec in self.kinds.items():
            ms, nb, fl, n = rec.totals()
            out[kind] = {"ms_per_step": ms / steps, "bytes_per_step": nb / steps, "flops_per_step": fl / steps,
                         "launches_per_step": n / steps}
        return out


_ACTIVE: Optional[StepRecorder] = None


def set_step_recorder(rec: Optional[StepRecorder]) -> None:
    global _ACTIVE
    _ACTIVE = rec


def step_recorder() -> Optional[StepRecorder]:
    return _ACTIVE


def begin():
    """An event recorded on the current stream, or ``None`` when no recorder is installed."""
    if _ACTIVE is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


def end(kind: str, ev0, nbytes: int, flops: int = 0) -> None:
    if ev0 is None or _ACTIVE is None:
        return
    ev1 = torch.cuda.Event(enable_timing=True)
    ev1.record()
    _ACTIVE.get(kind).records.append((ev0, ev1, int(nbytes), int(flops)))
