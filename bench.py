"""Benchmark of the Swin3D backbone hot path on B200.

Default (what the driver runs): the era5-shape Swin3D U-net backbone forward (benchmark config 4:
embed 512, encoder depths (6,10,8) / decoder (8,10,6), heads (8,16,32)/(32,16,8), window (2,6,12),
latent grid (4,180,360), batch 1) in the ``bf16_mixed`` tier, random init ~N(0, 0.02), synthetic
~N(0,1) input. One step = one backbone forward. Metric: ms/step (lower is better).

* ``value``      device time per step with the input resident in HBM (CUDA events, max over ranks);
                 the step is captured once as a CUDA graph and replayed.
* ``e2e``        the same steps through the public API from pinned host memory: every step's H2D
                 of its input and D2H of its full output are inside the timed region, overlapped
                 with the neighbouring steps' compute by ``flash_aurora_b200.pipeline.HostPipeline``.
* ``step_breakdown`` one eager pass of the same steps with CUDA events around every operator of
                 every block (partition, QKV GEMM, attention, proj GEMM, AdaLN1, fc1 + GELU, fc2,
                 AdaLN2): per operator its time per step, share, and achieved TFLOP/s or GB/s
                 against the measured peaks (GEMMs against the sustained bf16 figure, since they
                 run inside a long step). Library GEMMs are included.
* ``roofline``   the dominant kernel of this library in that breakdown, in the contract's form.
* ``gpu_launches`` kernel launches of this library inside the timed region, counted from the nodes
                 of the captured graph (``launches_per_step`` also gives the library ones).
* ``cpu_baseline`` the CPU oracle (upstream FP32 algorithm restated in torch-CPU) on one shifted
                 block per stage, extrapolated to the 48-block step (rank 0, N = 1 only).
* ``same_box_bars`` the stock PyTorch path on the same GPU, for comparison: config-2 attention
                 through ``scaled_dot_product_attention`` with the float mask, and one stage-1
                 block in eager PyTorch under bf16 autocast.

Multi-GPU (``torchrun --nproc-per-node N``): every rank runs its own backbone step on its own
input (independent ensemble members, no data-path collective): weak scaling, replicas. The
line also carries ``sharded_config5``: benchmark config 5 (a (4,360,720) x 512 Swin3D stage of
10 blocks) split into latitude bands across the N ranks with the NCCL point-to-point halo
exchange, strong scaling, with a parity check of the banded result against the whole field run on
one GPU (``--no-sharded`` skips it; ``--workload sharded`` runs it alone).

``--impl reference`` times the reference algorithm on the host CPU instead (the CPU oracle, see
above; rank 0 only) and prints the same metric. It cannot run a 48-block step within minutes, so
each timed "step" is one block and the line says so (``extrapolated``, ``blocks_timed``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "era5 Swin3D backbone ms/step (bf16_mixed)"
UNIT = "ms/step"
CONFIG4 = dict(embed_dim=512, encoder_depths=(6, 10, 8), encoder_num_heads=(8, 16, 32),
               decoder_depths=(8, 10, 6), decoder_num_heads=(32, 16, 8), window_size=(2, 6, 12))
PATCH_RES = (4, 180, 360)
TRAFFIC_RATIO = 0.973  # attention DRAM bytes / algorithmic bytes, ncu (profiles/attention_config2_tcgen05.md)
STAGES = [((4, 180, 360), 512, 8, 12), ((4, 90, 180), 1024, 16, 20), ((4, 45, 90), 2048, 32, 16)]


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _sustained_tflops() -> tuple[float, str]:
    """The bf16 GEMM peak under the power cap (seconds-long loop), for kernels timed in a step."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured sustained"
    except Exception:
        return 1400.0, "fallback sustained"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.proc = None
        ident = str(device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", ident,
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), ws, local
    return None, 0, 1, 0


def _max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------------------------
# CPU baseline: the upstream FP32 block algorithm restated on CPU (oracle), one shifted block per
# stage, extrapolated by block count.
# ----------------------------------------------------------------------------------------------
def _cpu_block_ms(res, dim, heads, seed):
    from oracle import block as OB
    from tests._inputs import block_param_shapes, init_params
    g = torch.Generator().manual_seed(seed)
    C, H, W = res
    x = torch.randn(1, C * H * W, dim, generator=g)
    c = torch.randn(1, 512, generator=g)
    shapes = block_param_shapes(dim, 512)
    p = init_params(shapes, seed=seed + 1)
    t0 = time.perf_counter()
    with torch.no_grad():
        OB.block_forward(x, c, res, p, num_heads=heads, window_size=(2, 6, 12), shift_size=(1, 3, 6))
    return (time.perf_counter() - t0) * 1e3


def cpu_baseline_sample() -> dict:
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    per = [_cpu_block_ms(res, dim, heads, 7 + i) for i, (res, dim, heads, _) in enumerate(STAGES)]
    total = sum(t * n for t, (_, _, _, n) in zip(per, STAGES))
    return {"value": round(total, 1), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": ("one shifted block per stage (S1 (4,180,360)x512, S2 (4,90,180)x1024, S3 (4,45,90)x2048) "
                       f"timed once each [{', '.join(f'{t:.0f}' for t in per)} ms], x(12,20,16) blocks; "
                       "stage merges/splits (1.4% of FLOPs) not timed")}


def run_reference(args) -> None:
    dist, rank, world, _ = (None, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    times = {0: [], 1: [], 2: []}
    for i in range(args.warmup + args.steps):
        s = i % 3
        res, dim, heads, _ = STAGES[s]
        ms = _cpu_block_ms(res, dim, heads, 7 + s)
        if i >= args.warmup:
            times[s].append(ms)
    for s in times:
        if not times[s]:
            res, dim, heads, _ = STAGES[s]
            times[s].append(_cpu_block_ms(res, dim, heads, 7 + s))
    value = sum(statistics.mean(times[s]) * STAGES[s][3] for s in range(3))
    blocks_timed = [len(times[s]) for s in range(3)]
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 1), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4: era5 Swin3D backbone forward, 48 blocks, grid (4,180,360), batch 1",
                   "parallelism": "host CPU"},
        # A 48-block FP32 step takes tens of minutes on the host; each timed "step" of this arm is
        # one shifted block of stage S1, S2, S3 in turn, and the value extrapolates the per-stage
        # mean to the step's (12, 20, 16) blocks. Stage merges/splits (1.4 % of FLOPs) are not timed.
        "extrapolated": True,
        "step_definition": "one shifted block of one stage (S1, S2, S3 in turn), not a backbone step",
        "blocks_timed": {"S1": blocks_timed[0], "S2": blocks_timed[1], "S3": blocks_timed[2]},
        "block_ms": {"S1": round(statistics.mean(times[0]), 1), "S2": round(statistics.mean(times[1]), 1),
                     "S3": round(statistics.mean(times[2]), 1)},
        "blocks_per_step": {"S1": STAGES[0][3], "S2": STAGES[1][3], "S3": STAGES[2][3]},
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "each step = one shifted block of stage S1/S2/S3 in turn on the CPU oracle "
                                   "(upstream FP32 algorithm), mean per stage x (12,20,16) blocks"},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------
# B200 arm
# ----------------------------------------------------------------------------------------------
# Operators of the block forward as the step recorder names them: (bound, implementation).
OPERATORS = {
    "partition": ("hbm", "this library: partition_kernel (first block of each stage)"),
    "qkv_gemm": ("tensor", "this library: tcgen05 GEMM, bias epilogue (CTA pair, 256 x 256 tiles)"),
    "attention": ("hbm", "this library: attn_tc_bf16_kernel (tcgen05)"),
    "proj_gemm": ("tensor", "this library: tcgen05 GEMM, bias epilogue (CTA pair, 256 x 256 tiles)"),
    "adaln1_unmerge": ("hbm", "this library: adaln_kernel (unmerge-fused, bf16 copy)"),
    "fc1_gelu_gemm": ("tensor", "this library: tcgen05 GEMM + GELU epilogue (CTA pair, 256 x 256 tiles)"),
    "fc2_gemm": ("tensor", "cuBLAS bf16 GEMM at stage 2, this library's CTA-pair GEMM at stage 3"),
    "adaln2_partition": ("hbm", "this library: adaln_kernel (next-partition fused)"),
    "adaln2": ("hbm", "this library: adaln_kernel"),
    "proj_adaln1": ("tensor+hbm", "this library: proj GEMM + unmerge + AdaLN1 + residual in one kernel (CTA pair)"),
    "fc2_adaln2": ("tensor+hbm", "this library: fc2 GEMM + AdaLN2 + residual (+ next partition) in one kernel (CTA pair)"),
}
# DRAM bytes / algorithmic bytes from ncu captures of the kernel (profiles/): the attention at
# config 2 and the fused fc1 + GELU at the config-4 stage-1 shape.
# fc1 + GELU at stage 1 on the CTA-pair kernel: 267.7 MB read + 1003 MB written against 1329 MB
# algorithmic (profiles/gemm_fc1_gelu_single_vs_pair_config4_s1.md; the single-CTA kernel, 0.956 too).
TRAFFIC_RATIOS = {"attention": TRAFFIC_RATIO, "fc1_gelu_gemm": 0.956}


def _is_own_kernel(name: str) -> bool:
    """Kernels of this library live in C++ namespace ``fa`` (mangled prefix ``_ZN2fa``)."""
    return name.startswith("_ZN2fa") or "fa::" in name


def step_breakdown(summary: dict, step_ms: float, hbm: float, tf_sus: float, tf_kind: str, peak_kind: str) -> list:
    rows = []
    for kind, v in sorted(summary.items(), key=lambda kv: -kv[1]["ms_per_step"]):
        bound, impl = OPERATORS.get(kind, ("hbm", "?"))
        ms = v["ms_per_step"]
        row = {"operator": kind, "impl": impl, "ms_per_step": round(ms, 3),
               "share_of_step": round(ms / step_ms, 3) if step_ms > 0 else None,
               "launches_per_step": round(v["launches_per_step"], 1), "bound": bound}
        if bound == "tensor":
            tf = v["flops_per_step"] / (ms * 1e-3) / 1e12 if ms > 0 else 0.0
            row.update({"achieved": round(tf, 1), "unit": "TFLOP/s", "peak": tf_sus, "peak_kind": tf_kind,
                        "frac": round(tf / tf_sus, 3)})
        elif bound == "tensor+hbm":
            # A GEMM whose epilogue carries a memory-bound op: both roofs, the higher fraction binds.
            tf = v["flops_per_step"] / (ms * 1e-3) / 1e12 if ms > 0 else 0.0
            gbs = v["bytes_per_step"] / (ms * 1e-3) / 1e9 if ms > 0 else 0.0
            row.update({"achieved": round(tf, 1), "unit": "TFLOP/s", "peak": tf_sus, "peak_kind": tf_kind,
                        "frac_tensor": round(tf / tf_sus, 3), "achieved_gbs": round(gbs, 1), "hbm_peak": hbm,
                        "frac_hbm": round(gbs / hbm, 3), "frac": round(max(tf / tf_sus, gbs / hbm), 3)})
        else:
            gbs = v["bytes_per_step"] / (ms * 1e-3) / 1e9 if ms > 0 else 0.0
            row.update({"achieved": round(gbs, 1), "unit": "GB/s", "peak": hbm, "peak_kind": peak_kind,
                        "frac": round(gbs / hbm, 3)})
        rows.append(row)
    return rows


def same_box_bars(dev) -> dict:
    """The stock PyTorch path on this GPU: config-2 attention through SDPA with the float mask,
    and one stage-1 shifted block in eager PyTorch under bf16 autocast (the upstream fallback
    path's operators: roll, pad, partition, Linear, SDPA, LayerNorm), each beside this library's."""
    import torch.nn.functional as F

    import flash_aurora_b200 as fa
    from flash_aurora_b200.swin3d import Swin3DTransformerBlock

    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    res, ws, ss = (4, 180, 360), (2, 6, 12), (1, 3, 6)
    Bwin, H, N, Dh = 1800, 8, 144, 64
    qkv = (torch.randn(Bwin, N, 3 * H * Dh, device=dev, generator=g) / 8.0).bfloat16()
    gids = fa.shifted_window_group_ids(res, ws, ss, device=dev)
    bias = torch.where(gids[:, :, None] != gids[:, None, :], -100.0, 0.0).to(torch.bfloat16)
    q, k, v = qkv.view(Bwin, N, 3, H, Dh).permute(2, 0, 3, 1, 4)
    ms_sdpa = _time_launches(lambda: F.scaled_dot_product_attention(q, k, v, attn_mask=bias[:, None]), 5,
                             flush=flush)
    ms_own = _time_launches(lambda: fa.window_attn_fwd_cute_qkvpacked(qkv, H, group_ids=gids, output_layout="bnc"),
                            5, flush=flush)
    del qkv, q, k, v, bias
    # One S1 shifted block.
    C, Hh, W = res
    D, heads = 512, 8
    blk = Swin3DTransformerBlock(dim=D, num_heads=heads, time_dim=D, window_size=ws, shift_size=ss).to(dev).eval()
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0.0, 0.02, generator=g) if p.ndim == 2 else p.zero_()
    x = torch.randn(1, C * Hh * W, D, device=dev, generator=g)
    c = torch.randn(1, D, device=dev, generator=g)
    mask = torch.where(gids[:, :, None] != gids[:, None, :], -100.0, 0.0)

    def eager_block():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            x5 = torch.roll(x.view(1, C, Hh, W, D), shifts=(-1, -3, -6), dims=(1, 2, 3))
            xw = x5.view(1, C // 2, 2, Hh // 6, 6, W // 12, 12, D).permute(0, 1, 3, 5, 2, 4, 6, 7).reshape(-1, N, D)
            qkv_ = F.linear(xw, blk.attn.qkv.weight, blk.attn.qkv.bias).view(-1, N, 3, heads, Dh).permute(2, 0, 3, 1, 4)
            a = F.scaled_dot_product_attention(qkv_[0], qkv_[1], qkv_[2], attn_mask=mask[:, None].to(qkv_.dtype))
            a = F.linear(a.transpose(1, 2).reshape(-1, N, D), blk.attn.proj.weight, blk.attn.proj.bias).float()
        a = a.view(1, C // 2, Hh // 6, W // 12, 2, 6, 12, D).permute(0, 1, 4, 2, 5, 3, 6, 7).reshape(1, C, Hh, W, D)
        a = torch.roll(a, shifts=(1, 3, 6), dims=(1, 2, 3)).reshape(1, -1, D)
        sh1, sc1 = blk.norm1.modulation(c)
        x1 = x + F.layer_norm(a, (D,)) * sc1 + sh1
        with torch.autocast("cuda", dtype=torch.bfloat16):
            hdn = F.gelu(F.linear(x1, blk.mlp.fc1.weight, blk.mlp.fc1.bias))
            hdn = F.linear(hdn, blk.mlp.fc2.weight, blk.mlp.fc2.bias)
        sh2, sc2 = blk.norm2.modulation(c)
        return x1 + F.layer_norm(hdn.float(), (D,)) * sc2 + sh2

    with torch.no_grad():
        ms_eager_blk = _time_launches(eager_block, 3, flush=flush)
        ms_own_blk = _time_launches(lambda: blk(x, c, res), 3, flush=flush)
    del blk, x, mask, flush
    torch.cuda.empty_cache()
    return {"attention_config2_masked_bf16": {"torch_sdpa_ms": round(ms_sdpa, 4), "this_library_ms": round(ms_own, 4),
                                              "speedup": round(ms_sdpa / ms_own, 2)},
            "block_s1_shifted_bf16": {"torch_eager_autocast_ms": round(ms_eager_blk, 3),
                                      "this_library_ms": round(ms_own_blk, 3),
                                      "speedup": round(ms_eager_blk / ms_own_blk, 2)},
            "note": "stock PyTorch operators on the same GPU (CUDA events, L2 flushed); the reference's own "
                    "CuTe/Triton kernels need their JIT sources at run time and are not on this box"}


def _bind_host_to_gpu(local: int) -> str:
    """Pin this rank's host threads to the CPUs NVML reports as closest to its GPU, so that the
    pinned host buffers of the end-to-end leg (allocated, and first touched, afterwards) sit on
    the GPU's own NUMA node. Only a process CPU mask changes; nothing on the GPU. Returns what was
    done, for the JSON line."""
    try:
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        if not cpus:
            return "not bound (NVML gave no CPUs)"
        os.sched_setaffinity(0, cpus)
        return f"bound to {len(cpus)} GPU-local CPUs"
    except Exception as exc:  # noqa: BLE001 - optional
        return f"not bound ({type(exc).__name__})"


def run_b200(args) -> None:
    from flash_aurora_b200 import recorder as R
    from flash_aurora_b200.status import check_device_status
    from flash_aurora_b200.swin3d import Swin3DTransformerBackbone, init_random_weights_

    dist, rank, world, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # Several ranks share the host: keep each one's copies on its GPU's NUMA node. A single rank
    # keeps every core (its CPU baseline uses them all).
    host_binding = _bind_host_to_gpu(local) if world > 1 else "not bound (one rank)"
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    model = Swin3DTransformerBackbone(**CONFIG4, precision="bf16_mixed").to(dev).eval()
    init_random_weights_(model, generator=gen)
    C, H, W = PATCH_RES
    L = C * H * W
    x = torch.randn(1, L, CONFIG4["embed_dim"], device=dev, generator=gen)
    lead = timedelta(hours=6)

    def step(inp):
        return model(inp, lead_time=lead, rollout_step=0, patch_res=PATCH_RES)

    with torch.no_grad():
        for _ in range(args.warmup):
            y = step(x)
        _barrier(dist)
        # The step runs as a captured CUDA graph (static shapes; flash_aurora_b200.graph).
        from flash_aurora_b200.graph import CapturedStep
        graphed = CapturedStep(step, x, warmup=1)
        for _ in range(args.warmup):
            graphed.replay()
        _barrier(dist)
        # Device-resident timing.
        sampler = ClockSampler(local)
        _barrier(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            y = graphed.replay()
        e1.record()
        _barrier(dist)
        clocks = sampler.stop()
        ms = e0.elapsed_time(e1) / args.steps
        ms = _max_over_ranks(dist, ms)
        check_device_status(dev)  # a kernel that gave up a bounded wait would raise here
        try:
            names = graphed.kernel_names()
            own = sum(1 for n in names if _is_own_kernel(n))
            launches = {"total": len(names), "this_library": own, "libraries": len(names) - own,
                        "source": "kernel nodes of the captured graph replayed in the timed region"}
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            launches = {"error": f"graph introspection failed: {exc}"}
        # Per-operator breakdown: the same steps run eagerly, with CUDA events around every
        # operator of every block on the launch stream (events cannot be timed inside a graph).
        srec = R.StepRecorder()
        R.set_step_recorder(srec)
        for _ in range(args.steps):
            step(x)
        torch.cuda.synchronize()
        R.set_step_recorder(None)
        summary = srec.summary(args.steps)
        attn_shapes = srec.get("attention").by_shape()

        # End to end from pinned host memory through the public API: every step uploads its
        # input and downloads its full output; HostPipeline overlaps those copies with the
        # neighbouring steps' compute (two host input and two host output buffers in rotation).
        # Two captures of the step (each with its own memory pool); each step uploads into its
        # slot's static input and downloads that slot's output directly: the skip half of the
        # final concatenation as soon as the first encoder layer has written it, the decoder half
        # after the replay.
        from flash_aurora_b200.graph import capture_backbone_slots
        from flash_aurora_b200.pipeline import HostPipeline
        slots = capture_backbone_slots(model, lead, 0, PATCH_RES, x, n=2, warmup=1)
        x_host = [x.cpu().pin_memory(), (x + 1.0).cpu().pin_memory()]
        out_host = [torch.empty(tuple(y.shape), dtype=y.dtype, pin_memory=True) for _ in range(2)]
        pipe = HostPipeline(slots, dev)
        pipe.run(x_host[:1], out_host[:1])  # warm the pipeline's streams and buffers
        pipe.wait()
        _barrier(dist)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record()
        pipe.run([x_host[i % 2] for i in range(args.steps)], [out_host[i % 2] for i in range(args.steps)])
        e3.record()
        _barrier(dist)
        pipe.wait()  # outputs landed; raises on a device-side failure
        e2e_ms = _max_over_ranks(dist, e2.elapsed_time(e3) / args.steps)
        yy = y

    hbm, _, peak_kind = _peaks()
    tf_sus, tf_kind = _sustained_tflops()
    rows = step_breakdown(summary, ms, hbm, tf_sus, tf_kind, peak_kind)
    # The contract's roofline object: the dominant kernel of this library in the breakdown.
    own_rows = [r for r in rows if r["impl"].startswith("this library")]
    top = max(own_rows, key=lambda r: r["ms_per_step"])
    tsum = summary[top["operator"]]
    n_top = tsum["launches_per_step"]
    per_launch_alg = (tsum["bytes_per_step"] / n_top) if n_top else None
    ratio = TRAFFIC_RATIOS.get(top["operator"])
    roofline = {"kernel": f"{top['operator']}: {top['impl']} (per-launch average over an eager pass of the same steps)",
                "bound": top["bound"], "achieved": top["achieved"], "peak": top["peak"], "unit": top["unit"],
                "frac": top["frac"], "peak_kind": top["peak_kind"],
                "traffic": round(ratio * per_launch_alg) if (ratio and per_launch_alg) else None,
                "traffic_source": "ncu DRAM bytes / algorithmic bytes of this kernel (profiles/) x this step's "
                                  "algorithmic bytes per launch" if ratio else None,
                "algorithmic_bytes_per_launch": round(per_launch_alg) if per_launch_alg else None,
                "flops_per_launch": round(tsum["flops_per_step"] / n_top) if n_top else None,
                "launches_per_step": n_top, "kernel_ms_per_step": top["ms_per_step"]}
    attn = summary.get("attention", {})
    n_blocks = sum(CONFIG4["encoder_depths"]) + sum(CONFIG4["decoder_depths"])
    line = {
        "metric": METRIC, "value": round(ms, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config4: era5 Swin3D U-net backbone forward (embed 512, depths (6,10,8)/(8,10,6), "
                               "heads (8,16,32)/(32,16,8), window (2,6,12), grid (4,180,360), batch 1), bf16_mixed",
                   "global_batch": world, "parallelism": f"replicas x{world} (independent members, no collective)",
                   "l2": "inputs and per-block activations > L2 (126 MB)",
                   "execution": "step captured once as a CUDA graph and replayed (static shapes)",
                   "blocks": n_blocks},
        "e2e": {"value": round(e2e_ms, 2), "unit": UNIT, "h2d_bytes_per_step": x.numel() * x.element_size(),
                "d2h_bytes_per_step": y.numel() * y.element_size(), "host_threads": host_binding},
        "gpu_launches": (launches["this_library"] * args.steps) if "this_library" in launches else None,
        "launches_per_step": launches,
        "roofline": roofline,
        "step_breakdown": rows,
        "attention_by_stage": [{"bytes": nb, "launches": n, "ms": round(t, 4),
                                "frac": round(nb / (t * 1e-3) / 1e9 / hbm, 3)} for nb, n, t in attn_shapes],
        "attention_tflops_in_step": round(attn["flops_per_step"] / (attn["ms_per_step"] * 1e-3) / 1e12, 1)
        if attn.get("ms_per_step") else None,
        "clocks": clocks,
    }
    del model, x, y, yy, graphed, pipe
    torch.cuda.empty_cache()
    if not args.no_sharded:
        line["sharded_config5"] = measure_sharded(dist, rank, world, local, min(args.steps, 5), 3)
    if rank == 0 and not args.no_bars:
        line["same_box_bars"] = same_box_bars(dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------------------------
# Config 5: a high-resolution Swin3D stage sharded by latitude bands across the ranks.
# ----------------------------------------------------------------------------------------------
CONFIG5 = dict(field=(4, 360, 720), dim=512, heads=8, depth=10, window=(2, 6, 12))


def measure_sharded(dist, rank, world, local, steps, warmup) -> dict:
    """Config 5 on ``world`` ranks: field (4,360,720) x 512, 8 heads, 10 blocks alternating
    unshifted/shifted, bf16_mixed; rank r holds latitude band r and exchanges its 3-row halo with
    its neighbours over NCCL for every shifted block. Strong scaling: the field is fixed."""
    from flash_aurora_b200.sharding import BandContext, halo_process_group
    from flash_aurora_b200.swin3d import BasicLayer3D

    dev = torch.device("cuda", local)
    cfg = CONFIG5
    C, H, W = cfg["field"]
    D = cfg["dim"]
    torch.manual_seed(4321)  # identical weights on every rank
    layer = BasicLayer3D(dim=D, depth=cfg["depth"], num_heads=cfg["heads"], ws=cfg["window"], time_dim=D,
                         precision="bf16_mixed")
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02)
    layer = layer.to(dev).eval()
    ctx = BandContext(cfg["field"], cfg["window"], rank, world, group=None, timeout_s=120)
    if dist is not None:
        # The world group, or with the overlapped exchanges (default from four ranks) their own group
        # with high-priority NCCL streams.
        group = halo_process_group(timeout_s=120) if ctx.overlap else dist.group.WORLD
        ctx = BandContext(cfg["field"], cfg["window"], rank, world, group=group, timeout_s=120)
    # Every rank draws the same whole field and keeps its band, so the banded result can be
    # checked against the whole field run unsharded on one GPU.
    gen = torch.Generator(device=dev).manual_seed(99)
    x_field = torch.randn(1, C, H, W, D, device=dev, generator=gen)
    Cb, Hb, Wb = ctx.res
    xb = x_field[:, :, ctx.h_begin:ctx.h_end].reshape(1, Cb * Hb * Wb, D).contiguous()
    c = torch.randn(1, D, device=dev, generator=torch.Generator(device=dev).manual_seed(98))
    with torch.no_grad():
        # Parity: this rank's band of the sharded stage against the same rows of the unsharded
        # stage (same weights, same input), reduced over the ranks.
        y_band, _ = layer(xb, c, ctx.res, band=ctx)
        y_full, _ = layer(x_field.reshape(1, C * H * W, D), c, cfg["field"])
        want = y_full.view(1, C, H, W, D)[:, :, ctx.h_begin:ctx.h_end].reshape_as(y_band)
        diff = (y_band.double() - want.double())
        acc = torch.stack([diff.square().sum(), want.double().square().sum()])
        mx = diff.abs().max().reshape(1)
        if dist is not None:
            dist.all_reduce(acc)
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        rel = float((acc[0] / acc[1]).sqrt().item())
        parity = {"rel_l2": rel, "max_abs": float(mx.item()), "bound": 5e-3, "ok": bool(rel <= 5e-3),
                  "against": "the same stage on the whole field, unsharded, on one GPU (same seeded weights "
                             "and input); bf16 GEMM rounding differs with the row count"}
        del y_full, want, diff, x_field
        torch.cuda.empty_cache()
        for _ in range(warmup):
            y, _ = layer(xb, c, ctx.res, band=ctx)
        ctx.wait()  # raises HaloExchangeError if a neighbour stopped answering
        _barrier(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            y, _ = layer(xb, c, ctx.res, band=ctx)
        e1.record()
        ctx.wait()
        _barrier(dist)
    ms = _max_over_ranks(dist, e0.elapsed_time(e1) / steps)
    shifted = cfg["depth"] // 2
    halo_fwd = C * 3 * W * D * 2 if world > 1 else 0  # rows to the previous band, sent as bf16
    halo_back = C * 3 * W * D * 2 if world > 1 else 0  # bf16 rows to the next band
    nw = C // 2 * (H // 6) * (W // 12)
    flops_block = 2 * C * H * W * D * (3 * D + D + 8 * D) + 4 * nw * cfg["heads"] * 144 * 144 * (D // cfg["heads"])
    del layer, xb, y, y_band
    torch.cuda.empty_cache()
    return {"workload": "config5: Swin3D stage, field (4,360,720) x 512, 8 heads, 10 blocks (5 shifted), "
                        "bf16_mixed, latitude bands of window rows, NCCL P2P 3-row halo per shifted block",
            "ms_per_step": round(ms, 3), "windows_per_s": round(nw * cfg["depth"] / (ms * 1e-3), 1),
            "tflops": round(flops_block * cfg["depth"] / (ms * 1e-3) / 1e12, 1),
            "bands": [list(b) for b in ctx.bounds], "scaling": "strong", "parity": parity,
            "halo_bytes_per_rank_per_step": shifted * (halo_fwd + halo_back),
            "halo_overlap": ("side stream, overlapped with the rows that need no halo" if ctx.overlap and world > 1
                             else "in line"),
            "steps": steps, "warmup": warmup}


def run_sharded(args) -> None:
    dist, rank, world, local = _dist()
    torch.cuda.set_device(local)
    out = measure_sharded(dist, rank, world, local, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------------------------
# Kernel-level workloads (benchmark configs 2 and 3); not the driver's default line.
# ----------------------------------------------------------------------------------------------
class L2Flush:
    """Empties L2 between timed launches: writes a 256 MB buffer (twice L2), then reads another
    256 MB buffer so that the flush's dirty lines are written back before the timed launch
    instead of during it."""

    def __init__(self, device) -> None:
        n = 256 * 1024 * 1024 // 4
        self.w = torch.empty(n, device=device)
        self.r = torch.zeros(n, device=device)
        self.sink = torch.empty((), device=device)

    def __call__(self) -> None:
        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.sink)


def _time_launches(fn, iters, warmup=3, flush=None):
    """Average device ms per call, CUDA events on the current stream, L2 flushed between calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    return total / iters


def run_attention(args) -> None:
    """Config 2: 1800 windows (grid (4,180,360), window (2,6,12)) x 8 heads x N=144 x d=64, packed
    QKV, shifted-window region mask, bf16 and fp32 (3xTF32) I/O."""
    import flash_aurora_b200 as fa
    dev = torch.device("cuda", 0)
    hbm, tflops_peak, kind = _peaks()
    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    res, ws, ss = (4, 180, 360), (2, 6, 12), (1, 3, 6)
    Bwin, H, N, Dh = 1800, 8, 144, 64
    gids = fa.shifted_window_group_ids(res, ws, ss, device=dev)
    flops = 4 * Bwin * H * N * N * Dh
    for dtype, label in ((torch.bfloat16, "bf16"), (torch.float32, "fp32_3xtf32")):
        qkv = (torch.randn(Bwin, N, 3 * H * Dh, device=dev, generator=g) / 8.0).to(dtype)
        out = torch.empty(Bwin, N, H * Dh, device=dev, dtype=dtype)
        for masked in (True, False):
            fn = lambda: fa.window_attn_fwd_cute_qkvpacked(qkv, H, group_ids=gids if masked else None,
                                                           output_layout="bnc", out=out)
            ms = _time_launches(fn, args.steps, flush=flush)
            nbytes = 4 * Bwin * H * N * Dh * qkv.element_size()
            gbs = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({
                "workload": f"config2 window attention {label} {'masked' if masked else 'unmasked'}",
                "ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                "tensor_peak_tflops": tflops_peak, "tensor_frac": round(flops / (ms * 1e-3) / 1e12 / tflops_peak, 3),
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(gbs / hbm, 3), "peak_kind": kind, "algorithmic_bytes": nbytes},
            }), flush=True)


def run_adaln_stages(args, flush=None) -> None:
    """AdaLN as the config-4 backbone launches it at each stage: norm1 fused with the window unmerge
    (bf16 windows in, fp32 residual and output, bf16 copy out) and norm2 fused with the next block's
    partition (bf16 x, fp32 residual and output, bf16 windows out): 12 bytes per element."""
    import flash_aurora_b200 as fa
    from flash_aurora_b200.adaln import adaptive_layernorm_film_add_residual_partition
    dev = torch.device("cuda", 0)
    hbm, _, kind = _peaks()
    flush = flush or L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    ws, ss = (2, 6, 12), (1, 3, 6)
    for tag, sres, sD in (("S1", (4, 180, 360), 512), ("S2", (4, 90, 180), 1024), ("S3", (4, 45, 90), 2048)):
        sL = sres[0] * sres[1] * sres[2]
        xs = torch.randn(1, *sres, sD, device=dev, generator=g)
        wins = fa.roll_pad_partition_windows(xs, sres, ws, ss, out_dtype=torch.bfloat16)
        del xs
        rs = torch.randn(1, sL, sD, device=dev, generator=g)
        hs = torch.randn(1, sL, sD, device=dev, generator=g).bfloat16()
        scs = torch.randn(1, 1, sD, device=dev, generator=g) * 0.1
        shs = torch.randn(1, 1, sD, device=dev, generator=g) * 0.1
        x1b = torch.empty(1, sL, sD, device=dev, dtype=torch.bfloat16)
        nxt = torch.zeros_like(wins)
        for name, fn in (
                ("norm1 unmerge + AdaLN + residual (+ bf16 copy)",
                 lambda: fa.unmerge_adaptive_layernorm_film_add_residual(wins, rs, scs, shs, sres, ws, ss, 0.0, 1e-5,
                                                                         out_bf16=x1b)),
                ("norm2 AdaLN + residual + next partition",
                 lambda: adaptive_layernorm_film_add_residual_partition(rs, hs, scs, shs, sres, ws, ss, nxt))):
            ms = _time_launches(fn, args.steps, flush=flush)
            nbytes = sL * sD * 12
            gbs = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({"workload": f"config4 {tag} {name} (L={sL}, D={sD})", "ms": round(ms, 4),
                              "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                           "frac": round(gbs / hbm, 3), "peak_kind": kind,
                                           "algorithmic_bytes": nbytes}}), flush=True)
        del wins, rs, hs, x1b, nxt


def run_layout_adaln(args) -> None:
    """Config 3 layout and AdaLN kernels (grid (4,45,90), D 2048, padded (4,48,96) -> 128 windows,
    shift (1,3,6)), then the config-4 per-stage AdaLN, GELU, Perceiver LN and fc1 + GELU launches."""
    import flash_aurora_b200 as fa
    dev = torch.device("cuda", 0)
    hbm, _, kind = _peaks()
    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    res, ws, ss = (4, 45, 90), (2, 6, 12), (1, 3, 6)
    C, H, W = res
    D = 2048
    L = C * H * W
    x = torch.randn(1, C, H, W, D, device=dev, generator=g)
    win = fa.roll_pad_partition_windows(x, res, ws, ss)
    branch = torch.randn(1, L, D, device=dev, generator=g).bfloat16()
    resid = torch.randn(1, L, D, device=dev, generator=g)
    scale = torch.randn(1, 1, D, device=dev, generator=g) * 0.1
    shift = torch.randn(1, 1, D, device=dev, generator=g) * 0.1
    nwin = win.shape[0] * win.shape[1]
    cases = [
        ("partition fp32->fp32", lambda: fa.roll_pad_partition_windows(x, res, ws, ss), L * D * 4 + nwin * D * 4),
        ("partition fp32->bf16", lambda: fa.roll_pad_partition_windows(x, res, ws, ss, out_dtype=torch.bfloat16),
         L * D * 4 + nwin * D * 2),
        ("unmerge fp32->fp32", lambda: fa.crop_roll_unmerge_windows(win, res, ws, ss), 2 * L * D * 4),
        ("adaln+residual bf16 x, fp32 residual -> fp32",
         lambda: fa.adaptive_layernorm_film_add_residual_forward(resid, branch, scale, shift, 0.0, output_fp32=True),
         L * D * (2 + 4 + 4)),
        ("unmerge+adaln+residual fp32 windows -> fp32",
         lambda: fa.unmerge_adaptive_layernorm_film_add_residual(win, resid, scale, shift, res, ws, ss),
         L * D * (4 + 4 + 4)),
    ]
    # The MLP activation at stage 1 of config 4: fc1 output (259200, 2048) bf16, in place.
    h = torch.randn(259200, 2048, device=dev, generator=g).bfloat16()
    cases.append(("mlp exact GELU (erfc form), S1 fc1 output (259200, 2048) bf16, in place",
                  lambda: fa.gelu_erf(h, inplace=True), h.numel() * 2 * 2))
    cases.append(("mlp exact GELU (erff, PyTorch arithmetic), same tensor",
                  lambda: fa.gelu_erf(h, inplace=True, method="erff"), h.numel() * 2 * 2))
    cases.append(("[torch F.gelu on the same tensor, for comparison]",
                  lambda: torch.nn.functional.gelu(h), h.numel() * 2 * 2))
    # The Perceiver level decoder's post-norm LayerNorm + residual at the era5 latent shape
    # (B*H*W = 259200 latents x 13 pressure levels, D = 512), bf16: x + residual read, out written.
    lat = torch.randn(259200, 13, 512, device=dev, generator=g).bfloat16()
    lat_res = torch.randn(259200, 13, 512, device=dev, generator=g).bfloat16()
    lw = torch.randn(512, device=dev, generator=g) * 0.1 + 1.0
    lb = torch.randn(512, device=dev, generator=g) * 0.1
    cases.append(("perceiver LayerNorm + residual, decoder latents (259200, 13, 512) bf16",
                  lambda: fa.layernorm_affine_add_residual_forward(lat, lat_res, lw, lb, 1e-5), lat.numel() * 2 * 3))
    cases.append(("[torch layer_norm + add on the same tensors, for comparison]",
                  lambda: torch.nn.functional.layer_norm(lat, (512,), lw.bfloat16(), lb.bfloat16(), 1e-5) + lat_res,
                  lat.numel() * 2 * 3))
    for name, fn, nbytes in cases:
        ms = _time_launches(fn, args.steps, flush=flush)
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"workload": f"config3 {name}", "ms": round(ms, 4),
                          "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                       "frac": round(gbs / hbm, 3), "peak_kind": kind, "algorithmic_bytes": nbytes}}),
              flush=True)
    del h, lat, lat_res, x, win, branch, resid
    run_adaln_stages(args, flush)
    # The block MLP's fc1 + GELU at each stage of config 4: fused tensor-core kernel vs cuBLAS + GELU.
    _, tf_peak, _ = _peaks()
    for tag, M, K, N in (("S1", 259200, 512, 2048), ("S2", 64800, 1024, 4096), ("S3", 16200, 2048, 8192)):
        a = torch.randn(M, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        b = (torch.randn(N, device=dev, generator=g) * 0.02).bfloat16()
        flops = 2 * M * N * K
        ms_f = _time_launches(lambda: fa.linear_bias_act(a, w, b, act="gelu"), args.steps, flush=flush)
        ms_c = _time_launches(lambda: fa.gelu_erf(torch.nn.functional.linear(a, w, b), inplace=True), args.steps,
                              flush=flush)
        tf = flops / (ms_f * 1e-3) / 1e12
        print(json.dumps({"workload": f"config4 {tag} fc1 + GELU fused (M={M}, K={K}, N={N})", "ms": round(ms_f, 4),
                          "unfused_cublas_plus_gelu_ms": round(ms_c, 4),
                          "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": tf_peak, "unit": "TFLOP/s",
                                       "frac": round(tf / tf_peak, 3), "peak_kind": kind}}), flush=True)
        del a, w, b


def run_gemm(args) -> None:
    """Every bf16 GEMM of the config-4 block at each stage (qkv, proj, fc1 + GELU, fc2): this
    library's single-CTA and CTA-pair tcgen05 kernels against cuBLAS (``F.linear``, + GELU for
    fc1), CUDA events, L2 flushed, TFLOP/s against the measured burst bf16 peak."""
    import flash_aurora_b200 as fa
    dev = torch.device("cuda", 0)
    _, tf_peak, kind = _peaks()
    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    shapes = []
    for tag, T, L, D in (("S1", 259200, 259200, 512), ("S2", 64800, 64800, 1024), ("S3", 18432, 16200, 2048)):
        shapes += [(tag, "qkv", T, D, 3 * D, "none"), (tag, "proj", T, D, D, "none"),
                   (tag, "fc1", L, D, 4 * D, "gelu"), (tag, "fc2", L, 4 * D, D, "none")]
    for tag, name, M, K, N, act in shapes:
        a = torch.randn(M, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        b = (torch.randn(N, device=dev, generator=g) * 0.02).bfloat16()
        flops = 2 * M * N * K
        res = {}
        for kernel in ("single", "pair"):
            os.environ["FA_GEMM_KERNEL"] = kernel
            res[kernel] = _time_launches(lambda: fa.linear_bias_act(a, w, b, act=act), args.steps, flush=flush)
        os.environ.pop("FA_GEMM_KERNEL", None)
        if act == "gelu":
            res["cublas"] = _time_launches(lambda: fa.gelu_erf(torch.nn.functional.linear(a, w, b), inplace=True),
                                           args.steps, flush=flush)
        else:
            res["cublas"] = _time_launches(lambda: torch.nn.functional.linear(a, w, b), args.steps, flush=flush)
        print(json.dumps({"workload": f"config4 {tag} {name} (M={M}, K={K}, N={N}, act={act})",
                          **{f"{k}_ms": round(v, 4) for k, v in res.items()},
                          **{f"{k}_tflops": round(flops / (v * 1e-3) / 1e12, 1) for k, v in res.items()},
                          "peak": tf_peak, "peak_kind": kind}), flush=True)
        del a, w, b
    run_fused_s1(args, flush, g)


def run_fused_s1(args, flush=None, g=None) -> None:
    """Stage 1 (D = 512): the fused linear + AdaLN kernel against the same linear on this library's
    GEMM followed by the stand-alone AdaLN kernel (unmerge-fused for proj, next-partition-fused for
    fc2), and against cuBLAS + AdaLN for fc2. A few GB on the device: small enough for an ncu
    capture of one launch."""
    import flash_aurora_b200 as fa
    from flash_aurora_b200.adaln import adaptive_layernorm_film_add_residual_partition
    from flash_aurora_b200.linear import linear_adaln_film_add_residual
    dev = torch.device("cuda", 0)
    flush = flush or L2Flush(dev)
    g = g or torch.Generator(device=dev).manual_seed(0)
    res, ws, ss = (4, 180, 360), (2, 6, 12), (1, 3, 6)
    L, D = 4 * 180 * 360, 512
    x = torch.randn(1, L, D, device=dev, generator=g)
    sc = torch.randn(1, 1, D, device=dev, generator=g) * 0.1
    sh = torch.randn(1, 1, D, device=dev, generator=g) * 0.1
    wins = torch.randn(1800, 144, D, device=dev, generator=g).bfloat16()
    wp = (torch.randn(D, D, device=dev, generator=g) * 0.02).bfloat16()
    bp = (torch.randn(D, device=dev, generator=g) * 0.02).bfloat16()
    xb = torch.empty(1, L, D, device=dev, dtype=torch.bfloat16)
    fused = _time_launches(lambda: linear_adaln_film_add_residual(wins, wp, bp, x, sc, sh, res, ws, ss, rows="windows",
                                                                  out_bf16=xb), args.steps, flush=flush)
    split = _time_launches(lambda: fa.unmerge_adaptive_layernorm_film_add_residual(
        fa.linear_bias_act(wins, wp, bp, act="none"), x, sc, sh, res, ws, ss, 0.0, 1e-5, out_bf16=xb),
        args.steps, flush=flush)
    print(json.dumps({"workload": "config4 S1 proj + unmerge + AdaLN1 + residual (+ bf16 copy)",
                      "fused_ms": round(fused, 4), "split_ms": round(split, 4)}), flush=True)
    del wins, wp, bp
    hid = torch.randn(1, L, 4 * D, device=dev, generator=g).bfloat16()
    w2 = (torch.randn(D, 4 * D, device=dev, generator=g) * 0.02).bfloat16()
    b2 = (torch.randn(D, device=dev, generator=g) * 0.02).bfloat16()
    nxt = torch.zeros(1800, 144, D, device=dev, dtype=torch.bfloat16)
    fused = _time_launches(lambda: linear_adaln_film_add_residual(hid, w2, b2, x, sc, sh, res, ws, (0, 0, 0),
                                                                  rows="tokens", next_windows=(ss, nxt)),
                           args.steps, flush=flush)
    split = _time_launches(lambda: adaptive_layernorm_film_add_residual_partition(
        x, fa.linear_bias_act(hid, w2, b2, act="none"), sc, sh, res, ws, ss, nxt), args.steps, flush=flush)
    cub = _time_launches(lambda: adaptive_layernorm_film_add_residual_partition(
        x, torch.nn.functional.linear(hid, w2, b2), sc, sh, res, ws, ss, nxt), args.steps, flush=flush)
    print(json.dumps({"workload": "config4 S1 fc2 + AdaLN2 + residual + next partition",
                      "fused_ms": round(fused, 4), "split_ms": round(split, 4), "split_cublas_ms": round(cub, 4)}),
          flush=True)
    from flash_aurora_b200.status import check_device_status
    check_device_status(dev)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="skip the config-5 sharded-stage object")
    ap.add_argument("--no-bars", action="store_true", help="skip the same-box stock PyTorch comparison")
    ap.add_argument("--workload", choices=["backbone", "attention", "layout_adaln", "adaln_stages", "sharded", "gemm",
                                           "fused_s1"],
                    default="backbone")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "attention":
        return run_attention(args)
    if args.workload == "layout_adaln":
        return run_layout_adaln(args)
    if args.workload == "adaln_stages":
        return run_adaln_stages(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload == "fused_s1":
        return run_fused_s1(args)
    if args.workload == "sharded" and args.impl != "reference":
        return run_sharded(args)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
