"""Generate the golden fixtures under ``tests/golden/`` from the upstream Flash-Aurora code.

Run in a container that has the upstream source tree::

    python tests/golden/make_golden.py --reference /path/to/Flash-Aurora [--only NAME ...]

It imports the upstream PyTorch modules unmodified (through ``_reference_shim``), runs them on
CPU in FP32 and writes compact ``.npz`` fixtures:

``layout_maps.npz``   source-index maps of the upstream roll/pad/partition and crop/roll/unmerge
                      (``swin3d.py`` pure-PyTorch path, the oracle of the upstream Triton test
                      ``tests/kernels/test_triton_swin3d.py:36-85``) for several geometries.
``mask_groups.npz``   per-window region ids taken from the upstream
                      ``compute_3d_shifted_window_mask`` image mask (``swin3d.py:526-599``).
``adaln.npz``         upstream ``AdaptiveLayerNorm`` forward / forward_add_residual outputs.
``attention.npz``     upstream ``WindowAttention`` (SDPA path with the real shifted mask).
``block_small.npz``   upstream ``Swin3DTransformerBlock`` (D=64, 1 head, grid (4,12,24)),
                      unshifted and shifted, full inputs/weights/outputs.
``block_config1.npz`` upstream block at config 1 (D=256, 4 heads, grid (4,36,72), shift
                      (1,3,6), seed 42): output checksums and a strided sample; inputs are
                      regenerated from the seed by ``tests/_inputs.py``.
``backbone_small.npz`` upstream ``Swin3DTransformerBackbone`` with odd stage sizes: output
                      checksums, a strided sample, and the upstream ``state_dict`` key list.
``backbone_config4.npz`` upstream backbone at config 4 (embed 512, depths (6,10,8)/(8,10,6),
                      grid (4,180,360), 48 blocks) in FP32: at each stage output of upstream's
                      error-accumulation trace, full-tensor checksums and 32 sampled token rows;
                      plus the drift of the oracle's ``bf16_mixed`` emulation (bf16 rounding
                      where upstream's tier rounds) against it, over the full tensors. Takes a
                      few minutes on 8 host cores.

The upstream default init zeroes the AdaLN modulation (film.py:45-48), which would make every
block an identity map; all Linear weights are therefore re-drawn ~N(0, 0.02) with zero biases
(``tests/_inputs.py:init_params``) before running.
"""

from __future__ import annotations

import argparse
import os
import sys
from datetime import timedelta

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import _reference_shim  # noqa: E402
from _inputs import (  # noqa: E402
    BACKBONE_CONFIG4,
    BACKBONE_SMALL,
    BLOCK_CONFIG1,
    TRACE_POINTS,
    BLOCK_SMALL,
    checksums,
    config1_inputs,
    config4_inputs,
    init_params,
    strided_sample,
    trace_rows,
)

LAYOUT_CASES = [
    # (name, res, window, shift)
    ("ref_test", (4, 8, 16), (2, 4, 4), (1, 2, 2)),
    ("ref_test_unshifted", (4, 8, 16), (2, 4, 4), (0, 0, 0)),
    ("config1", (4, 36, 72), (2, 6, 12), (1, 3, 6)),
    ("config1_unshifted", (4, 36, 72), (2, 6, 12), (0, 0, 0)),
    ("s3", (4, 45, 90), (2, 6, 12), (1, 3, 6)),
    ("s3_unshifted", (4, 45, 90), (2, 6, 12), (0, 0, 0)),
    ("odd_pad", (3, 13, 25), (2, 6, 12), (1, 3, 6)),
    ("small_res", (2, 5, 30), (2, 6, 12), (1, 3, 6)),
    ("tiny", (1, 6, 12), (2, 6, 12), (1, 3, 6)),
]

MASK_CASES = [
    ("ref_test", (4, 8, 16), (2, 4, 4), (1, 2, 2), True),
    ("config1", (4, 36, 72), (2, 6, 12), (1, 3, 6), True),
    ("config1_unwarped", (4, 36, 72), (2, 6, 12), (1, 3, 6), False),
    ("s1", (4, 180, 360), (2, 6, 12), (1, 3, 6), True),
    ("s2", (4, 90, 180), (2, 6, 12), (1, 3, 6), True),
    ("s3", (4, 45, 90), (2, 6, 12), (1, 3, 6), True),
    ("config5", (4, 360, 720), (2, 6, 12), (1, 3, 6), True),
    ("odd_pad", (3, 13, 25), (2, 6, 12), (1, 3, 6), True),
]
# Not a mask case: at res (2, 5, 30) the clamped windows give a 1x1xW window grid, and the
# upstream ``compute_3d_shifted_window_mask`` raises in ``mask_windows.view`` (swin3d.py:594,
# einops returns a non-contiguous view there). The layout maps above still cover that shape.


def _layout_maps(swin3d, util):
    out = {}
    for name, res, ws, ss in LAYOUT_CASES:
        C, H, W = res
        # Source index + 1 in float64 (exact), so 0 marks zero padding.
        x = (torch.arange(C * H * W, dtype=torch.float64) + 1).view(1, C, H, W, 1)
        wsa, ssa = util.maybe_adjust_windows(ws, ss, res)
        sx = torch.roll(x, shifts=(-ssa[0], -ssa[1], -ssa[2]), dims=(1, 2, 3)) if any(ssa) else x
        pad = ((-C) % wsa[0], (-H) % wsa[1], (-W) % wsa[2])
        sx = swin3d.pad_3d(sx, pad)
        win = swin3d.window_partition_3d(sx, wsa).reshape(-1, wsa[0] * wsa[1] * wsa[2])
        part = (win.long() - 1).to(torch.int32).numpy()
        # Inverse: slot index + 1 through window_reverse_3d -> crop_3d -> roll(+ss).
        nW, N = part.shape
        slots = (torch.arange(nW * N, dtype=torch.float64) + 1).view(nW, wsa[0], wsa[1], wsa[2], 1)
        merged = swin3d.window_reverse_3d(slots, wsa, sx.shape[1], sx.shape[2], sx.shape[3])
        merged = swin3d.crop_3d(merged, pad)
        if any(ssa):
            merged = torch.roll(merged, shifts=(ssa[0], ssa[1], ssa[2]), dims=(1, 2, 3))
        unm = (merged.reshape(-1).long() - 1).to(torch.int32).numpy()
        out[f"{name}/partition"] = part
        out[f"{name}/unmerge"] = unm
        out[f"{name}/spec"] = np.array([*res, *ws, *ss], dtype=np.int32)
    return out


def _mask_groups(swin3d, util):
    out = {}
    for name, res, ws, ss, warped in MASK_CASES:
        wsa, ssa = util.maybe_adjust_windows(ws, ss, res)
        _, img = swin3d.compute_3d_shifted_window_mask(
            res[0], res[1], res[2], wsa, ssa, torch.device("cpu"), torch.float32, warped=warped
        )
        win = swin3d.window_partition_3d(img, wsa).reshape(-1, wsa[0] * wsa[1] * wsa[2])
        out[f"{name}/groups"] = win.to(torch.uint8).numpy()
        out[f"{name}/spec"] = np.array([*res, *ws, *ss, int(warped)], dtype=np.int32)
    return out


def _adaln(film):
    torch.manual_seed(3)
    out = {}
    for tag, dim, ctx, L in (("d256", 256, 256, 64), ("d2048", 2048, 512, 4)):
        m = film.AdaptiveLayerNorm(dim, ctx).eval()
        with torch.no_grad():
            m.ln_modulation[1].weight.normal_(0.0, 0.02)
            m.ln_modulation[1].bias.normal_(0.0, 0.02)
        x = torch.randn(2, L, dim)
        xb = torch.randn(2, L, dim).bfloat16().float()
        res = torch.randn(2, L, dim)
        c = torch.randn(2, ctx)
        with torch.no_grad():
            shift, scale = m.ln_modulation(c).unsqueeze(1).chunk(2, dim=-1)
            y = m(x, c)
            yr = m.forward_add_residual(res, xb, c)
        out.update({
            f"{tag}/x": x.numpy(), f"{tag}/x_bf16_valued": xb.numpy(), f"{tag}/residual": res.numpy(),
            f"{tag}/shift": shift.numpy(), f"{tag}/scale": scale.numpy(),
            f"{tag}/forward": y.numpy(), f"{tag}/forward_add_residual": yr.numpy(),
        })
        if dim <= 256:  # the modulation Linear itself, only where it is small
            out.update({
                f"{tag}/c": c.numpy(), f"{tag}/w": m.ln_modulation[1].weight.detach().numpy(),
                f"{tag}/b": m.ln_modulation[1].bias.detach().numpy(),
            })
    return out


def _attention(swin3d):
    torch.manual_seed(5)
    res, ws, ss = (4, 12, 24), (2, 6, 12), (1, 3, 6)
    dim, heads = 128, 2
    m = swin3d.WindowAttention(dim, ws, heads).eval()
    with torch.no_grad():
        for lin in (m.qkv, m.proj):
            lin.weight.normal_(0.0, 0.02)
            lin.bias.normal_(0.0, 0.02)
    mask, _ = swin3d.compute_3d_shifted_window_mask(*res, ws, ss, torch.device("cpu"), torch.float32)
    nW = mask.shape[0]
    x = torch.randn(nW, 144, dim)
    with torch.no_grad():
        y_masked = m(x, mask=mask)
        y_plain = m(x, mask=None)
    return {
        "x": x.numpy(), "qkv_w": m.qkv.weight.detach().numpy(),
        "qkv_b": m.qkv.bias.detach().numpy(), "proj_w": m.proj.weight.detach().numpy(),
        "proj_b": m.proj.bias.detach().numpy(),
        "spec": np.array([*res, *ws, *ss, dim, heads], dtype=np.int32),
        "masked": y_masked.numpy(), "unmasked": y_plain.numpy(),
    }


def _block_small(swin3d):
    cfg = BLOCK_SMALL
    out = {}
    torch.manual_seed(cfg["seed"])
    C, H, W = cfg["res"]
    x = torch.randn(1, C * H * W, cfg["dim"])
    c = torch.randn(1, cfg["dim"])
    out["x"], out["c"] = x.numpy(), c.numpy()
    for tag, ss in (("unshifted", (0, 0, 0)), ("shifted", cfg["shift"])):
        blk = swin3d.Swin3DTransformerBlock(
            dim=cfg["dim"], num_heads=cfg["heads"], time_dim=cfg["dim"],
            window_size=cfg["window"], shift_size=ss,
        ).eval()
        sd = init_params({k: tuple(v.shape) for k, v in blk.state_dict().items()}, seed=cfg["seed"] + 1)
        blk.load_state_dict(sd)
        with torch.no_grad():
            y = blk(x, c, cfg["res"], 0)
        out[f"{tag}/y"] = y.numpy()
        for k, v in sd.items():
            out[f"{tag}/param/{k}"] = v.numpy()
    return out


def _block_config1(swin3d):
    cfg = BLOCK_CONFIG1
    blk = swin3d.Swin3DTransformerBlock(
        dim=cfg["dim"], num_heads=cfg["heads"], time_dim=cfg["dim"],
        window_size=cfg["window"], shift_size=cfg["shift"],
    ).eval()
    x, c, sd = config1_inputs({k: tuple(v.shape) for k, v in blk.state_dict().items()})
    blk.load_state_dict(sd)
    with torch.no_grad():
        y = blk(x, c, cfg["res"], 0)
    return {"checksums": checksums(y), "sample": strided_sample(y), "x_checksums": checksums(x)}


def _backbone_small(swin3d):
    cfg = BACKBONE_SMALL
    torch.manual_seed(cfg["seed"])
    bb = swin3d.Swin3DTransformerBackbone(
        embed_dim=cfg["embed_dim"], encoder_depths=cfg["encoder_depths"],
        encoder_num_heads=cfg["encoder_num_heads"], decoder_depths=cfg["decoder_depths"],
        decoder_num_heads=cfg["decoder_num_heads"], window_size=cfg["window"],
    ).eval()
    shapes = {k: tuple(v.shape) for k, v in bb.state_dict().items()}
    sd = init_params(shapes, seed=cfg["seed"] + 1)
    bb.load_state_dict(sd)
    C, H, W = cfg["patch_res"]
    g = torch.Generator().manual_seed(cfg["seed"] + 2)
    x = torch.randn(1, C * H * W, cfg["embed_dim"], generator=g)
    with torch.no_grad():
        y = bb(x, lead_time=timedelta(hours=6), rollout_step=0, patch_res=cfg["patch_res"])
    keys = sorted(shapes)
    return {
        "checksums": checksums(y), "sample": strided_sample(y), "out_shape": np.array(y.shape),
        "keys": np.array(keys), "key_shapes": np.array([str(shapes[k]) for k in keys]),
    }


def _diff(ref: torch.Tensor, cand: torch.Tensor) -> tuple[float, float]:
    """(relative L2, cosine similarity) in float64, as upstream's trace reports them
    (benchmark/bench_backbone_error_accum.py:117-132)."""
    r, c = ref.double().reshape(-1), cand.double().reshape(-1)
    rn = r.norm().item()
    return (c - r).norm().item() / rn, torch.dot(r, c).item() / (rn * c.norm().item())


def _backbone_config4(swin3d):
    """Upstream FP32 backbone at config 4 with the stage outputs captured by forward-pre-hooks
    on the stage modules (the input of each following stage is the previous stage's traced
    output), then the oracle's bf16_mixed emulation on the same inputs for the tier drift."""
    import time

    from oracle import block as OB

    cfg = BACKBONE_CONFIG4
    bb = swin3d.Swin3DTransformerBackbone(
        embed_dim=cfg["embed_dim"], encoder_depths=cfg["encoder_depths"],
        encoder_num_heads=cfg["encoder_num_heads"], decoder_depths=cfg["decoder_depths"],
        decoder_num_heads=cfg["decoder_num_heads"], window_size=cfg["window"],
    ).eval()
    shapes = {k: tuple(v.shape) for k, v in bb.state_dict().items()}
    x, sd = config4_inputs(shapes)
    bb.load_state_dict(sd)
    stages = list(bb.encoder_layers) + list(bb.decoder_layers)
    points: dict = {}

    def pre_hook(name):
        def hook(_mod, args):
            points[name] = args[0].detach().clone()
        return hook

    hooks = [stages[i + 1].register_forward_pre_hook(pre_hook(name))
             for i, name in enumerate(TRACE_POINTS[:-1])]
    t0 = time.perf_counter()
    with torch.no_grad():
        y = bb(x, lead_time=timedelta(hours=6), rollout_step=0, patch_res=cfg["patch_res"])
    for h in hooks:
        h.remove()
    points[TRACE_POINTS[-1]] = y
    print(f"upstream fp32 config-4 backbone: {time.perf_counter() - t0:.0f} s")
    del bb
    emu: dict = {}
    t0 = time.perf_counter()
    with torch.no_grad():
        OB.backbone_forward(x, timedelta(hours=6), cfg["patch_res"], sd, embed_dim=cfg["embed_dim"],
                            encoder_depths=cfg["encoder_depths"], encoder_num_heads=cfg["encoder_num_heads"],
                            decoder_depths=cfg["decoder_depths"], decoder_num_heads=cfg["decoder_num_heads"],
                            window_size=cfg["window"], bf16_mixed=True, trace=emu)
    print(f"oracle bf16_mixed emulation: {time.perf_counter() - t0:.0f} s")
    out = {"x_checksums": checksums(x), "points": np.array(TRACE_POINTS)}
    for name in TRACE_POINTS:
        t = points[name].reshape(-1, points[name].shape[-1])
        e = emu[name].reshape(t.shape)
        rows = trace_rows(t.shape[0], name)
        rel, cos = _diff(t, e)
        rel_rows, _ = _diff(t[rows], e[rows])
        out.update({
            f"{name}/checksums": checksums(t), f"{name}/shape": np.array(points[name].shape),
            f"{name}/row_index": rows.numpy(), f"{name}/rows": t[rows].numpy(),
            f"{name}/emulated_bf16_mixed": np.array([rel, cos, rel_rows]),
        })
        print(f"{name:>14}: emulated bf16_mixed drift rel-L2 {rel:.3e} (sampled rows {rel_rows:.3e}), "
              f"cos {cos:.8f}")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the upstream Flash-Aurora source tree")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*", default=None, help="fixture file names to (re)generate")
    args = ap.parse_args()
    _reference_shim.install(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from flash_aurora.aurora.model import film, swin3d, util

    jobs = {
        "layout_maps.npz": lambda: _layout_maps(swin3d, util),
        "mask_groups.npz": lambda: _mask_groups(swin3d, util),
        "adaln.npz": lambda: _adaln(film),
        "attention.npz": lambda: _attention(swin3d),
        "block_small.npz": lambda: _block_small(swin3d),
        "block_config1.npz": lambda: _block_config1(swin3d),
        "backbone_small.npz": lambda: _backbone_small(swin3d),
        "backbone_config4.npz": lambda: _backbone_config4(swin3d),
    }
    for fname, fn in jobs.items():
        if args.only is not None and fname not in args.only:
            continue
        data = fn()
        path = os.path.join(args.out, fname)
        np.savez_compressed(path, **data)
        print(f"wrote {path} ({os.path.getsize(path) / 1e3:.1f} kB)")


if __name__ == "__main__":
    main()
