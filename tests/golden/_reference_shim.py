"""Import shim for the upstream Flash-Aurora PyTorch modules (fixture generation only).

The upstream Swin3D block and AdaLN modules (``flash_aurora/aurora/model/swin3d.py``,
``flash_aurora/aurora/model/film.py``) import ``timm`` and the package ``__init__`` pulls in
the engine (``xarray``/``netCDF4``). None of those are installed here, so this shim:

* registers a minimal stand-in ``timm`` module providing ``to_2tuple``/``to_3tuple``,
  ``DropPath`` (identity at inference) and ``trunc_normal_`` (``torch.nn.init``);
* registers empty parent packages ``flash_aurora`` / ``flash_aurora.aurora`` /
  ``flash_aurora.aurora.model`` whose ``__path__`` points into the upstream tree, so that the
  submodules are imported straight from their upstream source files, unmodified.

This file is used by ``make_golden.py`` in the development container only; nothing under
``tests/`` that runs on a GPU box imports it.
"""

from __future__ import annotations

import os
import sys
import types


def install(reference_root: str) -> None:
    if "flash_aurora.aurora.model.swin3d" in sys.modules:
        return
    import torch

    timm = types.ModuleType("timm")
    layers = types.ModuleType("timm.layers")
    models = types.ModuleType("timm.models")
    vit = types.ModuleType("timm.models.vision_transformer")

    def _ntuple(n):
        def f(x):
            if isinstance(x, (tuple, list)):
                return tuple(x)
            return tuple([x] * n)

        return f

    class DropPath(torch.nn.Module):
        def __init__(self, p: float = 0.0) -> None:
            super().__init__()
            self.p = p

        def forward(self, x):
            return x

    layers.to_2tuple = _ntuple(2)
    layers.to_3tuple = _ntuple(3)
    layers.DropPath = DropPath
    vit.trunc_normal_ = torch.nn.init.trunc_normal_
    timm.layers = layers
    timm.models = models
    models.vision_transformer = vit
    sys.modules.update(
        {
            "timm": timm,
            "timm.layers": layers,
            "timm.models": models,
            "timm.models.vision_transformer": vit,
        }
    )

    pkg_root = os.path.join(reference_root, "flash_aurora")
    for name, sub in (
        ("flash_aurora", ""),
        ("flash_aurora.aurora", "aurora"),
        ("flash_aurora.aurora.model", os.path.join("aurora", "model")),
    ):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(pkg_root, sub)]
        sys.modules[name] = mod
