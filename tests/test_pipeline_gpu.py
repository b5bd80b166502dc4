"""HostPipeline: overlapped host I/O gives the same results as serial copies."""

from __future__ import annotations

import pytest
import torch

import flash_aurora_b200 as fa
from flash_aurora_b200.pipeline import HostPipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_matches_serial(depth):
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(depth)
    xs = [torch.randn(1 << 20, generator=g).pin_memory() for _ in range(7)]
    outs = [torch.empty(1 << 20, dtype=torch.bfloat16).pin_memory() for _ in range(7)]

    def step(t):
        y = (t * 3.0 + 1.0).to(torch.bfloat16)
        return fa.gelu_erf(y, inplace=True)

    HostPipeline(step, dev, depth=depth).run(xs, outs)
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        assert torch.equal(o, step(x.to(dev)).cpu())


def test_pipeline_reuses_output_buffers_in_order():
    dev = torch.device("cuda", 0)
    xs = [torch.full((4096,), float(i)).pin_memory() for i in range(6)]
    out = [torch.empty(4096).pin_memory() for _ in range(2)]
    HostPipeline(lambda t: t + 0.5, dev).run(xs, [out[i % 2] for i in range(6)])
    torch.cuda.synchronize()
    assert torch.equal(out[0], torch.full((4096,), 4.5)) and torch.equal(out[1], torch.full((4096,), 5.5))


def test_captured_backbone_step_matches_eager():
    """A backbone forward captured as a CUDA graph replays to the eager result, bit for bit, and the
    call form copies inputs in and outputs out."""
    from datetime import timedelta

    from flash_aurora_b200.graph import CapturedStep
    from flash_aurora_b200.swin3d import Swin3DTransformerBackbone, init_random_weights_

    dev = torch.device("cuda", 0)
    model = Swin3DTransformerBackbone(embed_dim=128, encoder_depths=(2, 2), encoder_num_heads=(2, 4),
                                      decoder_depths=(2, 2), decoder_num_heads=(4, 2), window_size=(2, 6, 12),
                                      precision="bf16_mixed").to(dev).eval()
    init_random_weights_(model, generator=torch.Generator(device=dev).manual_seed(3))
    res = (4, 24, 48)
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn(1, res[0] * res[1] * res[2], 128, device=dev, generator=g)
    step = lambda inp: model(inp, lead_time=timedelta(hours=6), rollout_step=0, patch_res=res)
    with torch.no_grad():
        want = step(x)
        graphed = CapturedStep(step, x)
        assert torch.equal(graphed.replay(), want)
        x2 = torch.randn(x.shape, device=dev, generator=g)
        assert torch.equal(graphed(x2), step(x2))
        assert torch.equal(graphed(x), want)


@pytest.mark.parametrize("n_slots", [1, 2, 3])
def test_captured_slots_pipeline_matches_eager(n_slots):
    """Captured slots: every step uploads into its slot, replays it and downloads its output;
    each host output equals the eager forward of its input, also when the host buffers rotate."""
    from datetime import timedelta

    from flash_aurora_b200.graph import capture_slots
    from flash_aurora_b200.swin3d import Swin3DTransformerBackbone, init_random_weights_

    dev = torch.device("cuda", 0)
    model = Swin3DTransformerBackbone(embed_dim=128, encoder_depths=(2, 2), encoder_num_heads=(2, 4),
                                      decoder_depths=(2, 2), decoder_num_heads=(4, 2), window_size=(2, 6, 12),
                                      precision="bf16_mixed").to(dev).eval()
    init_random_weights_(model, generator=torch.Generator(device=dev).manual_seed(5))
    res = (4, 24, 48)
    g = torch.Generator().manual_seed(6)
    xs = [torch.randn(1, res[0] * res[1] * res[2], 128, generator=g).pin_memory() for _ in range(5)]
    step = lambda inp: model(inp, lead_time=timedelta(hours=6), rollout_step=0, patch_res=res)
    with torch.no_grad():
        wants = [step(x.to(dev)).cpu() for x in xs]
        slots = capture_slots(step, xs[0].to(dev), n=n_slots)
        pipe = HostPipeline(slots, dev)
        outs = [torch.empty(tuple(wants[0].shape), pin_memory=True) for _ in range(5)]
        pipe.run(xs, outs)  # five steps through the slots in turn
        pipe.wait()
        for a, b in zip(outs, wants):
            assert torch.equal(a, b)
        rot = [torch.empty(tuple(wants[0].shape), pin_memory=True) for _ in range(2)]
        pipe.run(xs[::-1], [rot[i % 2] for i in range(5)])  # two host buffers in rotation
        pipe.wait()
    assert torch.equal(rot[0], wants[0]) and torch.equal(rot[1], wants[1])


def test_backbone_slots_download_the_skip_half_early():
    """Backbone slots: the skip half of every output leaves after the first encoder layer (an event
    recorded inside the graph), the decoder half after the replay; every host output equals the
    eager forward of its own input, bit for bit, over more steps than slots."""
    from datetime import timedelta

    from flash_aurora_b200.graph import capture_backbone_slots
    from flash_aurora_b200.swin3d import Swin3DTransformerBackbone, init_random_weights_

    dev = torch.device("cuda", 0)
    model = Swin3DTransformerBackbone(embed_dim=128, encoder_depths=(2, 2), encoder_num_heads=(2, 4),
                                      decoder_depths=(2, 2), decoder_num_heads=(4, 2), window_size=(2, 6, 12),
                                      precision="bf16_mixed").to(dev).eval()
    init_random_weights_(model, generator=torch.Generator(device=dev).manual_seed(7))
    res = (4, 24, 48)
    lead = timedelta(hours=6)
    g = torch.Generator().manual_seed(8)
    xs = [torch.randn(1, res[0] * res[1] * res[2], 128, generator=g).pin_memory() for _ in range(5)]
    with torch.no_grad():
        wants = [model(x.to(dev), lead_time=lead, rollout_step=0, patch_res=res).cpu() for x in xs]
        slots = capture_backbone_slots(model, lead, 0, res, xs[0].to(dev), n=2)
        assert model.skip_hook is None
        outs = [torch.full(tuple(wants[0].shape), float("nan")).pin_memory() for _ in range(5)]
        pipe = HostPipeline(slots, dev)
        pipe.run(xs, outs)
        pipe.wait()
    for a, b in zip(outs, wants):
        assert torch.equal(a, b)
