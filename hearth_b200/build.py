"""Builds the CUDA backend in-tree: hearth_b200/libhearth_b200.so (sm_100a only).

    python -m hearth_b200.build [--force]

nvcc flags: -gencode arch=compute_100a,code=sm_100a, -fmad=false (the reference's numerics forbid
contracted multiply-adds in canonical float math), -lineinfo for profiling, hidden visibility
except the C ABI of include/hearth_b200.h.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libhearth_b200.so")
SOURCES = ["hx_kernels.cu", "hx_decode.cu", "hx_prefill_tc.cu", "hx_capi.cu", "hx_store.cpp", "hx_noalloc.cu", "hx_container.cpp", "hx_model.cu"]
HEADERS = ["hx_common.cuh", "hx_device.cuh", "hx_kernels.h", "hx_store.h", "hx_route.cuh", "hx_moe_job.cuh", "hx_container.h",
           "hx_moe_internal.h"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-fmad=false", "-lineinfo",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-ffp-contract=off",
              "-shared"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(REPO, "include", "hearth_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc()] + NVCC_FLAGS + ["-o", tmp] + [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
