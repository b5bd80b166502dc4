"""Host-side behaviour of the Python mirror that needs no GPU: upstream error types, module
state-dict compatibility with the upstream backbone, workspace pool."""

from __future__ import annotations

import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200.swin3d import Swin3DTransformerBackbone, Swin3DTransformerBlock
from _inputs import BACKBONE_SMALL, block_param_shapes


def test_tf32_dtype_guard():
    q, k, v = (torch.randn(2, 4, 16, 16) for _ in range(3))
    with pytest.raises(AssertionError, match="float32"):
        fa.window_attn_fwd_cute(q.bfloat16(), k.bfloat16(), v.bfloat16(), precision=fa.WinAttnPrecision.TF32_ACC_FP32)


def test_bf16_mixed_dtype_guard():
    q, k, v = (torch.randn(2, 4, 16, 16) for _ in range(3))
    with pytest.raises(AssertionError, match="bfloat16"):
        fa.window_attn_fwd_cute(q, k, v, precision=fa.WinAttnPrecision.BF16_MIXED)


def test_dispatch_requires_cuda():
    q, k, v = (torch.randn(2, 4, 16, 16) for _ in range(3))
    with pytest.raises(RuntimeError, match="CUDA"):
        fa.window_attn_dispatch(q, k, v)


def test_layout_and_adaln_reject_cpu_tensors():
    x = torch.randn(1, 4, 8, 16, 32)
    with pytest.raises(ValueError, match="CUDA"):
        fa.roll_pad_partition_windows_triton(x, (4, 8, 16), (2, 4, 4), (1, 2, 2))
    with pytest.raises(ValueError, match="CUDA"):
        fa.crop_roll_unmerge_windows_triton(torch.randn(16, 32, 32), (4, 8, 16), (2, 4, 4), (1, 2, 2))
    with pytest.raises(ValueError, match="CUDA"):
        fa.adaptive_layernorm_film_forward(torch.randn(1, 4, 8), torch.randn(1, 1, 8), torch.randn(1, 1, 8), 0.0)
    with pytest.raises(ValueError, match="CUDA"):
        fa.adaptive_layernorm_film_add_residual_forward(torch.randn(1, 4, 8), torch.randn(1, 4, 8),
                                                        torch.randn(1, 1, 8), torch.randn(1, 1, 8), 0.0)


def test_qkvpacked_argument_errors():
    with pytest.raises(TypeError):
        fa.window_attn_fwd_cute_qkvpacked(torch.zeros(2, 144, 384, dtype=torch.float16), 2)
    with pytest.raises(ValueError, match="shape"):
        fa.window_attn_fwd_cute_qkvpacked(torch.zeros(144, 384), 2)
    with pytest.raises(ValueError, match="divisible"):
        fa.window_attn_fwd_cute_qkvpacked(torch.zeros(2, 144, 380), 2)
    with pytest.raises(ValueError, match="output_layout"):
        fa.window_attn_fwd_cute_qkvpacked(torch.zeros(2, 144, 384), 2, output_layout="nhd")


def test_block_state_dict_matches_upstream_keys():
    blk = Swin3DTransformerBlock(dim=256, num_heads=4, time_dim=256, window_size=(2, 6, 12), shift_size=(1, 3, 6))
    got = {k: tuple(v.shape) for k, v in blk.state_dict().items()}
    assert got == block_param_shapes(256, 256)


def test_backbone_state_dict_matches_upstream(golden):
    d = golden("backbone_small.npz")
    cfg = BACKBONE_SMALL
    bb = Swin3DTransformerBackbone(embed_dim=cfg["embed_dim"], encoder_depths=cfg["encoder_depths"],
                                   encoder_num_heads=cfg["encoder_num_heads"], decoder_depths=cfg["decoder_depths"],
                                   decoder_num_heads=cfg["decoder_num_heads"], window_size=cfg["window"])
    got = {k: str(tuple(v.shape)) for k, v in bb.state_dict().items()}
    want = dict(zip([str(k) for k in d["keys"]], [str(s) for s in d["key_shapes"]]))
    assert got == want


def test_block_forward_refuses_cpu():
    blk = Swin3DTransformerBlock(dim=64, num_heads=1, time_dim=64, window_size=(2, 6, 12))
    with pytest.raises(RuntimeError, match="CUDA"):
        blk(torch.randn(1, 4 * 12 * 24, 64), torch.randn(1, 64), (4, 12, 24))


def test_workspace_pool_reuses_buffers():
    pool = fa.InferenceWorkspacePool()
    a = pool.get("k", (2, 3), device="cpu", dtype=torch.float32)
    b = pool.get("k", (2, 3), device="cpu", dtype=torch.float32)
    c = pool.get("k", (2, 4), device="cpu", dtype=torch.float32)
    assert a.data_ptr() == b.data_ptr() and c.shape == (2, 4)
    # A smaller request of another dtype reuses the arena; a larger one grows it.
    d = pool.get("k", (3,), device="cpu", dtype=torch.bfloat16)
    assert d.data_ptr() == a.data_ptr() and d.dtype == torch.bfloat16
    big = pool.get("k", (1000,), device="cpu", dtype=torch.float32)
    assert big.numel() == 1000 and pool.nbytes() >= 4000
    other = pool.get("other", (2, 3), device="cpu", dtype=torch.float32)
    assert other.data_ptr() != big.data_ptr()
    assert pool.get("k", (0, 5), device="cpu", dtype=torch.float32).shape == (0, 5)
    pool.clear()
    assert pool.nbytes() == 0


def test_lead_time_expansion_matches_oracle():
    from datetime import timedelta  # noqa: F401
    from flash_aurora_b200.swin3d import lead_time_expansion
    from oracle.block import lead_time_expansion as ref
    h = torch.tensor([6.0, 0.5])
    torch.testing.assert_close(lead_time_expansion(h, 512), ref(h, 512), rtol=0, atol=0)


def test_kernel_recorder_groups_launches_by_size():
    """The per-stage view the backbone bench line reports: launches grouped by their algorithmic
    bytes, largest first, with the average time of each group (events faked on the host)."""
    from flash_aurora_b200.window_attn import KernelRecorder

    class Ev:
        def __init__(self, t):
            self.t = t

        def elapsed_time(self, other):
            return other.t - self.t

    rec = KernelRecorder()
    for nbytes, ms in ((300, 1.0), (900, 3.0), (300, 3.0), (600, 2.0), (900, 5.0)):
        rec.records.append((Ev(0.0), Ev(ms), nbytes, 4 * nbytes))
    assert rec.by_shape() == [(900, 2, 4.0), (600, 1, 2.0), (300, 2, 2.0)]
    total_ms, total_bytes, total_flops, launches = rec.totals()
    assert (total_ms, total_bytes, total_flops, launches) == (14.0, 3000, 12000, 5)


def test_maybe_adjust_windows_matches_oracle():
    """The package's window clamp equals the oracle's restatement of upstream util.py:54-72 (which
    the layout fixtures pin), including the assertion on a zero-sized axis."""
    import itertools

    from flash_aurora_b200.util import maybe_adjust_windows
    from oracle import layout as OL

    for res, ws, ss in itertools.product([(4, 45, 90), (2, 6, 12), (1, 5, 7), (3, 13, 25)],
                                         [(2, 6, 12), (4, 6, 12), (1, 1, 1)], [(0, 0, 0), (1, 3, 6)]):
        assert maybe_adjust_windows(ws, ss, res) == OL.maybe_adjust_windows(ws, ss, res)
    with pytest.raises(AssertionError, match="Window size must be positive"):
        maybe_adjust_windows((2, 6, 12), (1, 3, 6), (0, 6, 12))


def test_gating_predicates(monkeypatch):
    """The upstream ``can_use_*`` predicates (custom_op_paths.py:501-579) under their names: the
    upstream conditions plus the B200 kernels' own limits. On a CPU tensor every one is False;
    with the device check faked to pass, each condition is checked in turn."""
    from flash_aurora_b200 import custom_op_paths as cop

    x = torch.zeros(2, 144, 3 * 8 * 64)
    assert not cop.b200_available(x)
    assert not cop.can_use_triton_layout(x, enabled=True)
    assert not cop.can_use_cute_qkvpacked(x, num_heads=8, head_dim=64, cute_enabled=True, training=False,
                                          attn_dropout=0.0)
    monkeypatch.setattr(cop, "b200_available", lambda t: True)
    assert cop.can_use_triton_layout(x, enabled=True)
    assert not cop.can_use_triton_layout(x, enabled=False)
    assert not cop.can_use_triton_layout(x.half(), enabled=True)
    assert cop.can_use_triton_adaln(x, enabled=True, training=False, drop_path_is_identity=True)
    assert not cop.can_use_triton_adaln(x.bfloat16(), enabled=True, training=False, drop_path_is_identity=True)
    assert not cop.can_use_triton_adaln(x, enabled=True, training=True, drop_path_is_identity=True)
    assert cop.can_use_triton_gelu(x.bfloat16(), enabled=True, training=False, drop_p=0.0)
    assert not cop.can_use_triton_gelu(x, enabled=True, training=False, drop_p=0.1)
    ok = dict(num_heads=8, head_dim=64, cute_enabled=True, training=False, attn_dropout=0.0)
    with torch.no_grad():
        assert cop.can_use_cute_qkvpacked(x, **ok)
        assert cop.can_use_cute_qkvpacked(x.bfloat16(), **ok)
        assert not cop.can_use_cute_qkvpacked(x, **{**ok, "head_dim": 32})  # the kernels need 64
        assert not cop.can_use_cute_qkvpacked(x, **{**ok, "num_heads": 4})  # last dim != 3 * H * Dh
        assert not cop.can_use_cute_qkvpacked(x[:, :, : 3 * 8 * 64 - 1], **ok)
        assert not cop.can_use_cute_qkvpacked(x.transpose(0, 1), **ok)  # not contiguous
        assert not cop.can_use_cute_qkvpacked(torch.zeros(2, 160, 3 * 8 * 64), **ok)  # N > 144
        assert not cop.can_use_cute_qkvpacked(x, **{**ok, "attn_dropout": 0.1})
        assert cop.can_use_cute_window_attention(torch.zeros(2, 8, 144, 64), enabled=True, training=False,
                                                 attn_dropout=0.0)
    assert not cop.can_use_cute_qkvpacked(x, **ok)  # grad enabled
