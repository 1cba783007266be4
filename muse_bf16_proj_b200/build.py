"""Builds libmuse_proj.so in-tree with nvcc for sm_100a (the only target).

    python -m muse_bf16_proj_b200.build [--ptxas-verbose]

The library is a single CUDA translation unit (capi.cu, which includes the kernels) plus the host
codec (codec12.cpp), linked with the static CUDA runtime so it loads beside PyTorch's own.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libmuse_proj.so")
SOURCES = ["capi.cu", "codec12.cpp"]
HEADERS = ["ptx.cuh", "gather.cuh", "gemv.cuh", "gemv12t.cuh", "tc_tile.cuh", "tc_streamk.cuh", "tc_gemm.cuh",
           "tc_gemm2.cuh", "tc12.cuh", "tc_skinny.cuh", "router.cuh", "enc12.cuh", "enc12_core.h", "errors.h", "stream_read.cuh", "tc_rows.cuh", "tc_wide.cuh",
           "tc_pairk.cuh", "tc_pairsk.cuh", "gemv_tiles.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmuse_proj.so")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "muse_proj.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, ptxas_verbose: bool = False, out: str | None = None, defines=()) -> str:
    """Compiles the library (to `out` instead of the package's lib/ when given, with extra
    -D`defines`, e.g. for timing a variant side by side)."""
    target = out or LIB
    if out is None and not force and not _stale():
        return LIB
    os.makedirs(os.path.dirname(target), exist_ok=True)
    tmp = target + ".tmp"
    cmd = [nvcc_path(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O3",
           "-o", tmp] + [f"-D{d}" for d in defines] + [os.path.join(CSRC, s) for s in SOURCES] + ["-lpthread"]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if ptxas_verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    print(build(force=True, ptxas_verbose="--ptxas-verbose" in sys.argv))
