"""Register budgets of the kernels, checked at compile time (no GPU).

The row kernels are tuned with `__launch_bounds__` so that their vector paths keep every value in
registers. Unbounded, ptxas chose 40 registers for the fp32 -> fp32 layout copies and spilled
24-36 bytes, which cost them 6-8 % of their bandwidth. The 3xTF32 attention moves registers
between warpgroups with `setmaxnreg`. These tests compile the sources for sm_100a with
`-Xptxas -v` and fail if a tuned instantiation spills again.
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

CSRC = os.path.join(ROOT, "flash_aurora_b200", "csrc")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"

pytestmark = pytest.mark.skipif(not os.path.exists(NVCC), reason="nvcc not available")


def _ptxas_report(source: str, tmp_path) -> dict[str, tuple[int, int]]:
    """{mangled kernel name: (registers, spill-store bytes)} for every entry of `source`."""
    out = subprocess.run(
        [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xptxas", "-v",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-c", os.path.join(CSRC, source),
         "-o", str(tmp_path / "k.o")],
        capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    report: dict[str, tuple[int, int]] = {}
    name, spill = None, 0
    for line in out.stderr.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            name, spill = m.group(1), 0
            continue
        m = re.search(r"(\d+) bytes spill stores", line)
        if m and name:
            spill = int(m.group(1))
        m = re.search(r"Used (\d+) registers", line)
        if m and name:
            report[name] = (int(m.group(1)), spill)
            name = None
    return report


def test_layout_kernels_do_not_spill(tmp_path):
    report = _ptxas_report("layout.cu", tmp_path)
    kernels = {k: v for k, v in report.items() if "partition_kernel" in k or "unmerge_kernel" in k}
    assert len(kernels) >= 12, sorted(kernels)
    spilled = {k: v for k, v in kernels.items() if v[1] > 0}
    assert not spilled, spilled


def test_adaln_vector_kernels_do_not_spill(tmp_path):
    report = _ptxas_report("adaln.cu", tmp_path)
    # Vector-path instantiations carry `Lb1E` (kVec = true) in their mangled names.
    vec = {k: v for k, v in report.items() if "adaln_kernel" in k and "Lb1E" in k}
    assert len(vec) >= 8, sorted(vec)
    spilled = {k: v for k, v in vec.items() if v[1] > 0}
    assert not spilled, spilled
    # D <= 512 rows are held to 64 registers (four 256-thread blocks per SM).
    small = {k: v for k, v in vec.items() if re.search(r"Lb1ELi[12]E", k)}
    assert small and all(r <= 64 for r, _ in small.values()), small


def test_fused_gemm_does_not_spill(tmp_path):
    report = _ptxas_report("gemm.cu", tmp_path)
    kernels = {k: v for k, v in report.items() if "gemm_bias_act_kernel" in k or "gemm_pair_bias_act_kernel" in k}
    assert len(kernels) == 4, sorted(kernels)
    spilled = {k: v for k, v in kernels.items() if v[1] > 0}
    assert not spilled, spilled


def test_gemm_adaln_register_budget(tmp_path):
    """320 threads are allocated registers as 384 (whole warpgroups): 168 per thread. The
    token-row variant keeps everything in registers; the window-row variant (slot -> token index
    arithmetic for four rows at a time) may spill a few words."""
    report = _ptxas_report("gemm_adaln.cu", tmp_path)
    kernels = {k: v for k, v in report.items() if "gemm_adaln_pair_kernel" in k}
    assert len(kernels) == 2, sorted(kernels)
    assert all(regs <= 168 for regs, _ in kernels.values()), kernels
    tokens = {k: v for k, v in kernels.items() if "ILi0EE" in k}
    assert tokens and all(spill == 0 for _, spill in tokens.values()), kernels
    assert all(spill <= 16 for _, spill in kernels.values()), kernels


def test_attention_kernels_register_budget(tmp_path):
    report = _ptxas_report("attention.cu", tmp_path)

    def variants(kind: str, masks: tuple[int, ...]) -> dict[str, tuple[int, int]]:
        pat = re.compile(rf"attn_tc_{kind}_kernelILi({'|'.join(str(m) for m in masks)})ELb[01]E")
        return {k: v for k, v in report.items() if pat.search(k)}

    # bf16: unmasked and region-id masks (the backbone's launches) keep everything in registers.
    bf16 = variants("bf16", (0, 1, 3))
    assert len(bf16) == 6, sorted(bf16)
    assert all(spill == 0 for _, spill in bf16.values()), bf16
    # 3xTF32, full-N unmasked and region-mask variants: the per-warpgroup register split holds
    # the softmax spills to a few words (60-72 bytes without it).
    tf32 = {k: v for k, v in variants("tf32", (0, 1)).items() if "Lb1E" in k}
    assert len(tf32) == 2, sorted(tf32)
    assert all(spill <= 24 for _, spill in tf32.values()), tf32
