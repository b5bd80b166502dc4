"""Seeded synthetic inputs and weights shared by the fixture generator and the tests.

Everything is drawn on the CPU with ``torch.Generator`` so that the same call sequence gives
bit-identical tensors here and on a GPU box (same image, same torch version).
"""

from __future__ import annotations

import numpy as np
import torch

# Config 1 of the benchmark plan: one shifted Swin3D block, FP32, runs on CPU.
BLOCK_CONFIG1 = dict(dim=256, heads=4, res=(4, 36, 72), window=(2, 6, 12), shift=(1, 3, 6), seed=42)
# A small block whose full inputs, weights and outputs fit in a fixture.
BLOCK_SMALL = dict(dim=64, heads=1, res=(4, 12, 24), window=(2, 6, 12), shift=(1, 3, 6), seed=7)
# A small U-net backbone with odd stage sizes (merge padding, split cropping, clamped windows).
BACKBONE_SMALL = dict(
    embed_dim=128, encoder_depths=(2, 2, 2), encoder_num_heads=(2, 4, 8),
    decoder_depths=(2, 2, 2), decoder_num_heads=(8, 4, 2), window=(2, 6, 12),
    patch_res=(4, 30, 60), seed=11,
)
# Config 4 of the benchmark plan: the era5-shape backbone (48 blocks, latent grid (4,180,360)).
BACKBONE_CONFIG4 = dict(
    embed_dim=512, encoder_depths=(6, 10, 8), encoder_num_heads=(8, 16, 32),
    decoder_depths=(8, 10, 6), decoder_num_heads=(32, 16, 8), window=(2, 6, 12),
    patch_res=(4, 180, 360), seed=2024,
)
# Stage outputs recorded along the backbone, named as upstream's error-accumulation trace names
# them (benchmark/bench_backbone_error_accum.py:180-216): each encoder stage after its patch
# merge, the first decoder stage, the additive-skip sum of the middle one and the final
# concatenation (the backbone output).
TRACE_POINTS = ("enc0_out", "enc1_out", "enc2_out", "dec0_out", "dec1_skip_add", "dec2_concat")
TRACE_ROWS = 32


def init_params(shapes: dict, seed: int, weight_std: float = 0.02, bias_std: float = 0.0) -> dict:
    """Re-draw a Swin3D state dict: 2-D weights ~N(0, std), biases ~N(0, bias_std) (0 by
    default), 1-D LayerNorm weights = 1. Keys are visited in sorted order."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for k in sorted(shapes):
        shp = tuple(shapes[k])
        if k.endswith(".weight") and len(shp) == 2:
            out[k] = torch.randn(shp, generator=g) * weight_std
        elif k.endswith(".weight"):
            out[k] = torch.ones(shp)
        elif k.endswith(".bias"):
            out[k] = torch.randn(shp, generator=g) * bias_std if bias_std else torch.zeros(shp)
        else:
            raise KeyError(f"unexpected parameter {k}")
    return out


def config1_inputs(shapes: dict):
    """x ~N(0,1) (1, 10368, 256), c ~N(0,1) (1, 256), weights ~N(0, 0.02), biases 0; seed 42."""
    cfg = BLOCK_CONFIG1
    g = torch.Generator().manual_seed(cfg["seed"])
    C, H, W = cfg["res"]
    x = torch.randn(1, C * H * W, cfg["dim"], generator=g)
    c = torch.randn(1, cfg["dim"], generator=g)
    return x, c, init_params(shapes, seed=cfg["seed"] + 1)


def block_param_shapes(dim: int, ctx: int, mlp_ratio: float = 4.0) -> dict:
    """Upstream ``Swin3DTransformerBlock`` state-dict keys and shapes (swin3d.py:655-681)."""
    hid = int(dim * mlp_ratio)
    return {
        "norm1.ln_modulation.1.weight": (2 * dim, ctx), "norm1.ln_modulation.1.bias": (2 * dim,),
        "attn.qkv.weight": (3 * dim, dim), "attn.qkv.bias": (3 * dim,),
        "attn.proj.weight": (dim, dim), "attn.proj.bias": (dim,),
        "norm2.ln_modulation.1.weight": (2 * dim, ctx), "norm2.ln_modulation.1.bias": (2 * dim,),
        "mlp.fc1.weight": (hid, dim), "mlp.fc1.bias": (hid,),
        "mlp.fc2.weight": (dim, hid), "mlp.fc2.bias": (dim,),
    }


def checksums(t: torch.Tensor) -> np.ndarray:
    d = t.double()
    return np.array([d.sum().item(), d.abs().sum().item(), (d * d).sum().item(),
                     d.max().item(), d.min().item()], dtype=np.float64)


def config4_inputs(shapes: dict):
    """Config-4 weights (``init_params``, seed 2025) and input x ~N(0,1) (1, 259200, 512) (seed
    2026), both drawn on the CPU."""
    cfg = BACKBONE_CONFIG4
    params = init_params(shapes, seed=cfg["seed"] + 1)
    C, H, W = cfg["patch_res"]
    g = torch.Generator().manual_seed(cfg["seed"] + 2)
    x = torch.randn(1, C * H * W, cfg["embed_dim"], generator=g)
    return x, params


def trace_rows(n_tokens: int, name: str, rows: int = TRACE_ROWS) -> torch.Tensor:
    """The sorted token rows sampled at trace point ``name``: a fixed draw per point name."""
    seed = sum((i + 1) * ord(ch) for i, ch in enumerate(name))
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(n_tokens, generator=g)[:rows].sort().values


def strided_sample(t: torch.Tensor, n: int = 4096) -> np.ndarray:
    flat = t.reshape(-1)
    step = max(1, flat.numel() // n)
    return flat[::step].numpy().astype(np.float32)
