"""Named output buffers that fixed-shape inference reuses from call to call.

The layout ops accept ``pool=`` (the upstream keyword, with keys such as ``"partition"`` and
``"unmerge"``) so that a forecast loop does not allocate its window tensors on every block call.

Storage here is one raw byte arena per (name, device), grown when a request needs more bytes and
otherwise reused: asking for a name again with the same shape and dtype returns a tensor over the
same memory, and asking for a smaller or differently typed tensor of the same name reuses the
arena too (no allocation), which keeps a stage sequence of different shapes at its high-water
mark. A returned tensor aliases every other tensor handed out under the same name and device:
callers treat it as scratch that the next request of that name overwrites.
"""

from __future__ import annotations

import math

import torch

__all__ = ["InferenceWorkspacePool"]

_ALIGN = 256  # byte alignment of every arena (covers 16-byte vector and TMA base requirements)


def _device_of(device) -> torch.device:
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


class InferenceWorkspacePool:
    """``get(name, shape, device=..., dtype=...)`` -> a tensor backed by the arena of ``name``."""

    def __init__(self) -> None:
        self._arenas: dict[tuple[str, torch.device], torch.Tensor] = {}

    def get(self, key: str, shape, *, device, dtype: torch.dtype) -> torch.Tensor:
        dev = _device_of(device)
        shape = tuple(int(s) for s in shape)
        itemsize = torch.empty((), dtype=dtype).element_size()
        need = math.prod(shape) * itemsize
        arena = self._arenas.get((key, dev))
        if arena is None or arena.numel() < need:
            # Round the capacity up so that small growth does not reallocate every call.
            cap = max(_ALIGN, -(-need // _ALIGN) * _ALIGN)
            arena = torch.empty(cap, dtype=torch.uint8, device=dev)
            self._arenas[(key, dev)] = arena
        return arena[:need].view(dtype).view(shape)

    def nbytes(self) -> int:
        """Bytes held by all arenas."""
        return sum(a.numel() for a in self._arenas.values())

    def clear(self) -> None:
        """Drop every arena (tensors already handed out keep their memory alive)."""
        self._arenas.clear()
