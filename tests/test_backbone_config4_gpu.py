"""Parity at the benchmarked backbone size (config 4): the 48-block era5-shape backbone (embed 512,
depths (6,10,8)/(8,10,6), grid (4,180,360)) with the seeded weights and input of
``tests/_inputs.py``, against the upstream FP32 backbone run on the CPU
(``tests/golden/backbone_config4.npz``, made by ``make_golden.py``).

At each stage output of upstream's error-accumulation trace (benchmark/bench_backbone_error_accum.py:
180-216) the fixture holds 32 sampled token rows and full-tensor checksums. Bounds:

* FP32 tier (strict FP32 GEMMs, 3xTF32 attention): relative L2 <= 1e-5 per stage output on the
  sampled rows, and the full-tensor norm within 1e-5;
* ``bf16_mixed``: the tier drift (relative L2 against upstream FP32 on the sampled rows) must stay
  within the drift of upstream's own ``bf16_mixed`` rounding, emulated by the oracle (bf16 where
  upstream's autocast rounds) over the same 48 blocks: at most 1.25x that drift, and the cosine
  similarity of the sampled rows at least 0.9999.
"""

from __future__ import annotations

import math
from datetime import timedelta

import numpy as np
import pytest
import torch

from flash_aurora_b200.swin3d import Swin3DTransformerBackbone
from _inputs import BACKBONE_CONFIG4, TRACE_POINTS, config4_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def config4_run(golden):
    d = golden("backbone_config4.npz")
    cfg = BACKBONE_CONFIG4
    bb = Swin3DTransformerBackbone(embed_dim=cfg["embed_dim"], encoder_depths=cfg["encoder_depths"],
                                   encoder_num_heads=cfg["encoder_num_heads"], decoder_depths=cfg["decoder_depths"],
                                   decoder_num_heads=cfg["decoder_num_heads"], window_size=cfg["window"],
                                   precision="fp32")
    shapes = {k: tuple(v.shape) for k, v in bb.state_dict().items()}
    x, sd = config4_inputs(shapes)
    bb.load_state_dict(sd)
    del sd
    bb = bb.cuda().eval()
    x = x.cuda()
    stages = list(bb.encoder_layers) + list(bb.decoder_layers)
    out = {}
    for precision in ("fp32", "bf16_mixed"):
        bb.set_precision(precision)
        points: dict = {}

        def pre_hook(name):
            def hook(_mod, args):
                t = args[0].reshape(-1, args[0].shape[-1])
                points[name] = (t[torch.from_numpy(d[f"{name}/row_index"]).cuda()].double().cpu(),
                                t.double().square().sum().item())
            return hook

        hooks = [stages[i + 1].register_forward_pre_hook(pre_hook(name))
                 for i, name in enumerate(TRACE_POINTS[:-1])]
        with torch.no_grad():
            y = bb(x, timedelta(hours=6), 0, cfg["patch_res"])
        for h in hooks:
            h.remove()
        t = y.reshape(-1, y.shape[-1])
        points[TRACE_POINTS[-1]] = (t[torch.from_numpy(d[f"{TRACE_POINTS[-1]}/row_index"]).cuda()].double().cpu(),
                                    t.double().square().sum().item())
        out[precision] = points
        del y, t
    return d, out


def _drift(got: torch.Tensor, want: np.ndarray) -> tuple[float, float]:
    w = torch.from_numpy(want).double()
    rel = ((got - w).norm() / w.norm()).item()
    cos = (torch.dot(got.reshape(-1), w.reshape(-1)) / (got.norm() * w.norm())).item()
    return rel, cos


@pytest.mark.parametrize("name", TRACE_POINTS)
def test_fp32_tier_matches_upstream(config4_run, name):
    d, out = config4_run
    rows, sumsq = out["fp32"][name]
    rel, _ = _drift(rows, d[f"{name}/rows"])
    assert rel <= 1e-5, f"{name}: fp32 tier rel-L2 {rel:.3e}"
    norm_ref = math.sqrt(d[f"{name}/checksums"][2])
    assert abs(math.sqrt(sumsq) - norm_ref) / norm_ref <= 1e-5


@pytest.mark.parametrize("name", TRACE_POINTS)
def test_bf16_mixed_within_upstream_tier_drift(config4_run, name):
    d, out = config4_run
    rows, _ = out["bf16_mixed"][name]
    rel, cos = _drift(rows, d[f"{name}/rows"])
    emu_full, emu_cos, emu_rows = (float(v) for v in d[f"{name}/emulated_bf16_mixed"])
    print(f"{name}: bf16_mixed drift rel-L2 {rel:.4e} cos {cos:.8f}; upstream tier (emulated) "
          f"{emu_rows:.4e} on the same rows, {emu_full:.4e} over the full tensor")
    assert rel <= 1.25 * emu_rows, f"{name}: drift {rel:.3e} vs emulated upstream tier {emu_rows:.3e}"
    assert cos >= 0.9999
