"""Build the in-tree CUDA library ``libflash_aurora_b200.so`` for sm_100a with nvcc.

``python -m flash_aurora_b200.build`` (or ``build()``) compiles every ``csrc/*.cu`` into one
shared object next to this file. The C ABI is declared in ``include/flash_aurora_b200.h``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libflash_aurora_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-O3", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, extra: list[str]) -> str:
    os.makedirs(OBJ, exist_ok=True)
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(INCLUDE, "flash_aurora_b200.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps) and not extra:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if extra:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    extra = list(extra or [])
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources()))
    if (not os.path.exists(LIB) or extra
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            # The driver library is resolved at run time; link against the toolkit stub here.
            stub = "/usr/local/cuda/lib64/stubs"
            cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-L", stub, "-lcuda"]
            r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    extra = ["-Xptxas", "-v"] if "-v" in sys.argv else None
    build(verbose=True, extra=extra)
