"""Keyed reusable output buffers for fixed-shape inference.

Same interface as upstream ``flash_aurora/aurora/model/workspace_pool.py:24-53``: ``get``
returns the cached tensor for ``key`` when shape, dtype and device match, otherwise allocates.
"""

from __future__ import annotations

from typing import Optional

import torch

__all__ = ["InferenceWorkspacePool"]


def _normalize_device(device) -> torch.device:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        return torch.device("cuda", torch.cuda.current_device())
    return d


class InferenceWorkspacePool:
    """Keyed buffers reused when ``(key, shape, device, dtype)`` match."""

    def __init__(self) -> None:
        self._buffers: dict[str, torch.Tensor] = {}

    def get(self, key: str, shape: tuple[int, ...], *, device, dtype: torch.dtype) -> torch.Tensor:
        device = _normalize_device(device)
        t: Optional[torch.Tensor] = self._buffers.get(key)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device:
            t = torch.empty(shape, device=device, dtype=dtype)
            self._buffers[key] = t
        return t

    def clear(self) -> None:
        self._buffers.clear()
