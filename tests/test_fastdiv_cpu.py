"""The multiply-and-shift division of the layout index maps (``FastDiv`` in csrc/fa_common.cuh),
checked on the host against integer division: the header's own ``make_fastdiv`` / ``fdiv``,
compiled by nvcc for the CPU (no GPU needed), over every divisor up to 4096, the divisors the
geometries use, and numerators at the edges of the 31-bit range."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import ROOT

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
pytestmark = pytest.mark.skipif(not os.path.exists(NVCC), reason="nvcc not available")

_PROGRAM = r"""
#include <cstdio>
#include <cstdint>
#include "fa_common.cuh"

static uint64_t state = 88172645463325252ull;
static uint32_t next_u31() {
  state ^= state << 13; state ^= state >> 7; state ^= state << 17;
  return (uint32_t)(state >> 33);
}

static int check(int64_t d, int32_t n, long* bad) {
  const fa::FastDiv f = fa::make_fastdiv(d);
  if (fa::fdiv(n, f) != (int32_t)(n / d)) {
    if (*bad < 5) std::printf("mismatch d=%lld n=%d got=%d\n", (long long)d, n, fa::fdiv(n, f));
    ++*bad;
  }
  return 0;
}

int main() {
  long bad = 0, n_checks = 0;
  const int32_t edges[] = {0, 1, 2, 3, 1023, 1024, 65535, 65536, 1 << 30, (1 << 30) + 1,
                           0x7ffffffe, 0x7fffffff};
  const int64_t big[] = {1 << 20, (1 << 20) + 1, 259200, 1036800, 2073600, 3 * (1 << 28),
                         (1ll << 30) - 1, 1ll << 30, (1ll << 30) + 1, 0x7ffffffe, 0x7fffffff};
  for (int64_t d = 1; d <= 4096; ++d) {
    for (int32_t n : edges) { check(d, n, &bad); ++n_checks; }
    for (int i = 0; i < 200; ++i) { check(d, (int32_t)next_u31(), &bad); ++n_checks; }
    for (int32_t k = 0; k < 4; ++k) {  // around multiples of d
      const int64_t m = (int64_t)(next_u31() / d) * d;
      for (int64_t n = m - 1; n <= m + 1; ++n)
        if (n >= 0 && n < (1ll << 31)) { check(d, (int32_t)n, &bad); ++n_checks; }
    }
  }
  for (int64_t d : big) {
    for (int32_t n : edges) { check(d, n, &bad); ++n_checks; }
    for (int i = 0; i < 100000; ++i) { check(d, (int32_t)next_u31(), &bad); ++n_checks; }
  }
  std::printf("checks=%ld bad=%ld\n", n_checks, bad);
  return bad != 0;
}
"""


def test_fastdiv_matches_integer_division(tmp_path):
    src = tmp_path / "fastdiv_check.cu"
    src.write_text(_PROGRAM)
    exe = tmp_path / "fastdiv_check"
    build = subprocess.run(
        [NVCC, "-std=c++17", "-O2", "-I" + os.path.join(ROOT, "include"),
         "-I" + os.path.join(ROOT, "flash_aurora_b200", "csrc"), str(src), "-o", str(exe)],
        capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-2000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout[-2000:]
    assert "bad=0" in run.stdout
