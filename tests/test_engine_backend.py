"""The reference engine with the B200 binding (oracle/_ref/libhearth_cuda.so) on the CPU side: built
from the reference's own sources plus oracle/hearth_cuda_backend.c, it exports the unchanged public
API, evaluates exactly like the unchanged reference while HEARTH_BACKEND is unset, and, when the
backend is asked for but no GPU can take it, fails every evaluation instead of falling back to the
CPU. Where the reference checkout is present, its own Python toolkit (python/hearth/engine.py) drives
the library unchanged through HEARTH_LIB."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tests.engine_util import CUDA_LIB, FIXTURE, REF_LIB, Engine, session

pytestmark = pytest.mark.skipif(not (os.path.exists(CUDA_LIB) and os.path.exists(REF_LIB)),
                                reason="oracle/_ref not built (needs the reference checkout)")

PROMPT = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3]


def test_binding_exports_the_public_api_only():
    out = subprocess.run(["nm", "-D", "--defined-only", CUDA_LIB], capture_output=True, text=True).stdout
    names = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    for sym in ("hearth_open", "hearth_eval", "hearth_close", "hearth_trace_start", "hearth_route_replay"):
        assert sym in names
    assert not any(n.startswith("hxc_") for n in names)   # the binding's own functions stay internal


def test_backend_off_evaluates_like_the_reference(monkeypatch):
    monkeypatch.delenv("HEARTH_BACKEND", raising=False)
    with Engine(REF_LIB) as a, Engine(CUDA_LIB) as b:
        la = session(a, PROMPT, 4)
        lb = session(b, PROMPT, 4)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_backend_requested_without_a_gpu_fails_instead_of_falling_back(monkeypatch):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present: the GPU tests cover the backend")
    except ImportError:
        pass
    monkeypatch.setenv("HEARTH_BACKEND", "cuda")
    with Engine(CUDA_LIB) as e:
        rc, _ = e.eval(PROMPT)
        assert rc == -4                       # HX_E_IO: the MoE layers cannot run where they were asked to
        rc, _ = e.eval(PROMPT)
        assert rc == -4                       # and stay refused: no CPU fallback


def test_reference_toolkit_drives_the_binding(monkeypatch):
    ref = O.reference_tree()
    if not ref:
        pytest.skip("the reference checkout is not present")
    code = f"""
import sys, numpy as np
sys.path.insert(0, {os.path.join(ref, 'python')!r})
from hearth.engine import Engine
e = Engine({FIXTURE!r}, cache_gb=0.05, threads=2, direct_io=False)
np.save(sys.argv[1], e.eval({PROMPT!r}, all_logits=True))
"""
    outs = []
    for lib in (REF_LIB, CUDA_LIB):
        env = dict(os.environ, HEARTH_LIB=lib)
        env.pop("HEARTH_BACKEND", None)
        path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"hx_toolkit_{os.getpid()}_{len(outs)}.npy")
        r = subprocess.run([sys.executable, "-c", code, path], env=env, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        outs.append(np.load(path))
        os.unlink(path)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
