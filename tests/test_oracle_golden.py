"""Pin the CPU oracle against fixtures produced by the upstream Flash-Aurora code itself."""

from __future__ import annotations

from datetime import timedelta

import numpy as np
import pytest
import torch

from oracle import block as OB
from oracle import layout as OL
from _inputs import BACKBONE_SMALL, BLOCK_CONFIG1, BLOCK_SMALL, block_param_shapes, checksums, config1_inputs, init_params, strided_sample


def _cases(d, suffix):
    return sorted({k.split("/")[0] for k in d if k.endswith(suffix)})


def test_layout_maps_match_upstream(golden):
    d = golden("layout_maps.npz")
    names = _cases(d, "/spec")
    assert len(names) >= 8
    for name in names:
        spec = d[f"{name}/spec"]
        res, ws, ss = tuple(spec[:3]), tuple(spec[3:6]), tuple(spec[6:9])
        g = OL.geometry(res, ws, ss)
        np.testing.assert_array_equal(OL.partition_source_index(g), d[f"{name}/partition"], err_msg=name)
        np.testing.assert_array_equal(OL.unmerge_source_index(g), d[f"{name}/unmerge"], err_msg=name)


def test_layout_apply_roundtrip_is_identity():
    rng = np.random.default_rng(0)
    for res, ws, ss in (((4, 8, 16), (2, 4, 4), (1, 2, 2)), ((3, 13, 25), (2, 6, 12), (1, 3, 6))):
        x = rng.standard_normal((2, *res, 8)).astype(np.float32)
        w = OL.roll_pad_partition(x, res, ws, ss)
        np.testing.assert_array_equal(OL.crop_roll_unmerge(w, res, ws, ss), x)


def test_mask_groups_match_upstream(golden):
    d = golden("mask_groups.npz")
    names = _cases(d, "/spec")
    assert "config5" in names and "s3" in names
    for name in names:
        spec = d[f"{name}/spec"]
        res, ws, ss, warped = tuple(spec[:3]), tuple(spec[3:6]), tuple(spec[6:9]), bool(spec[9])
        got = OL.window_group_ids(res, ws, ss, warped)
        np.testing.assert_array_equal(got, d[f"{name}/groups"], err_msg=name)


def test_mask_counts_match_survey_figures():
    # Windows that hold more than one region id under the real shifted mask, at the config 1,
    # stage-1, stage-3 and config 5 grids.
    for res, expect in (((4, 36, 72), 42), ((4, 180, 360), 930), ((4, 45, 90), 103), ((4, 360, 720), 3660)):
        gid = OL.window_group_ids(res, (2, 6, 12), (1, 3, 6))
        masked = int((gid != gid[:, :1]).any(axis=1).sum())
        assert masked == expect, (res, masked)


def test_adaln_matches_upstream(golden):
    d = golden("adaln.npz")
    for tag in ("d256", "d2048"):
        t = {k.split("/", 1)[1]: torch.from_numpy(v) for k, v in d.items() if k.startswith(tag + "/")}
        y = OB.adaln(t["x"], t["shift"], t["scale"])
        torch.testing.assert_close(y, t["forward"], rtol=1e-6, atol=1e-6)
        yr = t["residual"] + OB.adaln(t["x_bf16_valued"], t["shift"], t["scale"])
        torch.testing.assert_close(yr, t["forward_add_residual"], rtol=1e-6, atol=1e-6)
        if "w" in t:
            p = {"n.ln_modulation.1.weight": t["w"], "n.ln_modulation.1.bias": t["b"]}
            sh, sc = OB.adaln_modulation(t["c"], p, "n.")
            torch.testing.assert_close(sh, t["shift"], rtol=1e-6, atol=1e-6)
            torch.testing.assert_close(sc, t["scale"], rtol=1e-6, atol=1e-6)


def test_window_attention_matches_upstream(golden):
    d = golden("attention.npz")
    spec = d["spec"]
    res, ws, ss, dim, heads = tuple(spec[:3]), tuple(spec[3:6]), tuple(spec[6:9]), int(spec[9]), int(spec[10])
    p = {"a.qkv.weight": torch.from_numpy(d["qkv_w"]), "a.qkv.bias": torch.from_numpy(d["qkv_b"]),
         "a.proj.weight": torch.from_numpy(d["proj_w"]), "a.proj.bias": torch.from_numpy(d["proj_b"])}
    x = torch.from_numpy(d["x"])
    mask = torch.from_numpy(OL.shifted_window_mask(res, ws, ss))
    torch.testing.assert_close(OB.window_attention(x, mask, p, "a.", heads), torch.from_numpy(d["masked"]), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(OB.window_attention(x, None, p, "a.", heads), torch.from_numpy(d["unmasked"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tag", ["unshifted", "shifted"])
def test_block_small_matches_upstream(golden, tag):
    d = golden("block_small.npz")
    cfg = BLOCK_SMALL
    p = {k.split("/param/", 1)[1]: torch.from_numpy(v) for k, v in d.items() if k.startswith(tag + "/param/")}
    ss = (0, 0, 0) if tag == "unshifted" else cfg["shift"]
    y = OB.block_forward(torch.from_numpy(d["x"]), torch.from_numpy(d["c"]), cfg["res"], p,
                         num_heads=cfg["heads"], window_size=cfg["window"], shift_size=ss)
    torch.testing.assert_close(y, torch.from_numpy(d[f"{tag}/y"]), rtol=1e-5, atol=1e-5)


def test_block_config1_matches_upstream(golden):
    d = golden("block_config1.npz")
    cfg = BLOCK_CONFIG1
    x, c, p = config1_inputs(block_param_shapes(cfg["dim"], cfg["dim"]))
    np.testing.assert_allclose(checksums(x), d["x_checksums"], rtol=1e-12)
    y = OB.block_forward(x, c, cfg["res"], p, num_heads=cfg["heads"], window_size=cfg["window"], shift_size=cfg["shift"])
    np.testing.assert_allclose(strided_sample(y), d["sample"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(checksums(y)[1:3], d["checksums"][1:3], rtol=1e-6)


def test_backbone_small_matches_upstream(golden):
    d = golden("backbone_small.npz")
    cfg = BACKBONE_SMALL
    shapes = {k: tuple(int(s) for s in v.strip("()").split(",") if s.strip()) for k, v in zip(d["keys"], d["key_shapes"])}
    p = init_params(shapes, seed=cfg["seed"] + 1)
    C, H, W = cfg["patch_res"]
    g = torch.Generator().manual_seed(cfg["seed"] + 2)
    x = torch.randn(1, C * H * W, cfg["embed_dim"], generator=g)
    y = OB.backbone_forward(x, timedelta(hours=6), cfg["patch_res"], p, embed_dim=cfg["embed_dim"],
                            encoder_depths=cfg["encoder_depths"], encoder_num_heads=cfg["encoder_num_heads"],
                            decoder_depths=cfg["decoder_depths"], decoder_num_heads=cfg["decoder_num_heads"],
                            window_size=cfg["window"])
    assert tuple(y.shape) == tuple(d["out_shape"])
    np.testing.assert_allclose(strided_sample(y), d["sample"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(checksums(y)[1:3], d["checksums"][1:3], rtol=1e-5)
