"""Builds the host-side test helper libraries of tests/native (test support only)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build_expf_check() -> str:
    out = os.path.join(HERE, "libexpf_check.so")
    src = os.path.join(HERE, "expf_check.cu")
    hdr = os.path.join(HERE, "..", "..", "hearth_b200", "csrc", "hx_common.cuh")
    if os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(src), os.path.getmtime(hdr)):
        return out
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
           "-Xcompiler", "-pthread", "-shared", "-o", out, src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(r.stdout + r.stderr)
    return out
