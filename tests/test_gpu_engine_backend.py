"""End to end through the reference engine's own public API with the B200 binding: the same container
and tokens evaluated by the reference engine on the CPU and by the engine built with
oracle/hearth_cuda_backend.c with HEARTH_BACKEND=cuda give bit-identical logits for every prompt and
decode position and byte-identical routing traces (docs/FORMAT.md §9 files written by
hearth_trace_start), both with the whole forward on the GPU (embedding, attention and KV cache, MoE
and dense layers, LM head) and with only the MoE layers there (HEARTH_CUDA_SCOPE=moe): the GPU is
pinned by the engine itself rather than by a restatement. Also with an expert cache smaller than the
container (HEARTH_CUDA_CACHE_GB), and with the prompt split into several forward calls (max_batch)."""
import os

import numpy as np
import pytest

from tests.engine_util import CUDA_LIB, REF_LIB, Engine, session

pytestmark = pytest.mark.gpu

PROMPT = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3]


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("scope", ["full", "moe"])
@pytest.mark.parametrize("model,cache_gb,max_batch", [("tiny_moe", None, 0), ("tiny_moe", "0.0001", 0),
                                                      ("tiny_moe", None, 5), ("tiny_qwen3_moe", None, 0),
                                                      ("tiny_olmoe", None, 3), ("tiny_qwen2_moe", "0.0001", 0),
                                                      ("tiny_deepseek_v3", None, 0)])
def test_gpu_backend_gives_the_reference_engines_logits_and_trace(gpu, monkeypatch, tmp_path, model, cache_gb,
                                                                   max_batch, scope):
    """scope full: the whole forward on the GPU; moe: the MoE layers only (HEARTH_CUDA_SCOPE=moe). An MLA
    container (tiny_deepseek_v3) takes the MoE-only scope either way."""
    path = os.path.join(GOLDEN, model + ".hearth")
    monkeypatch.delenv("HEARTH_BACKEND", raising=False)
    with Engine(REF_LIB, model=path, max_batch=max_batch) as cpu:
        want = session(cpu, PROMPT, 8, str(tmp_path / "cpu.trace"))
    monkeypatch.setenv("HEARTH_BACKEND", "cuda")
    if scope == "moe":
        monkeypatch.setenv("HEARTH_CUDA_SCOPE", "moe")
    if cache_gb:
        monkeypatch.setenv("HEARTH_CUDA_CACHE_GB", cache_gb)   # the store's minimum: E + 2 slots, streaming
    with Engine(CUDA_LIB, model=path, max_batch=max_batch) as gpu_engine:
        got = session(gpu_engine, PROMPT, 8, str(tmp_path / "gpu.trace"))
    assert np.isfinite(want).all()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    a = open(tmp_path / "cpu.trace", "rb").read()
    b = open(tmp_path / "gpu.trace", "rb").read()
    assert len(a) > 0 and a == b


def test_gpu_backend_on_a_device_that_does_not_exist_fails(gpu, monkeypatch):
    monkeypatch.setenv("HEARTH_BACKEND", "cuda")
    monkeypatch.setenv("HEARTH_CUDA_DEVICE", "97")
    with Engine(CUDA_LIB) as e:
        rc, _ = e.eval(PROMPT)
    assert rc == -4


@pytest.mark.parametrize("scope", ["full", "moe"])
def test_gpu_route_replay_gives_the_reference_engines_logits(gpu, monkeypatch, tmp_path, scope):
    """hearth_route_replay with the backend: the replayed ids (a trace recorded from another prompt)
    drive the GPU's MoE layers (hxb_moe_forward_routed) exactly as they drive moe_layer on the CPU."""
    monkeypatch.delenv("HEARTH_BACKEND", raising=False)
    trace = str(tmp_path / "rec.trace")
    with Engine(REF_LIB) as rec:
        session(rec, PROMPT[::-1], 6, trace)
    other = [7, 2, 7, 1, 8, 2, 8, 1, 8, 2]
    with Engine(REF_LIB) as cpu:
        plain = session(cpu, other, 4)
    with Engine(REF_LIB) as cpu:
        assert cpu.route_replay(trace) == 0
        want = session(cpu, other, 4)
    assert not np.array_equal(want, plain)   # the replay changed the routing
    monkeypatch.setenv("HEARTH_BACKEND", "cuda")
    if scope == "moe":
        monkeypatch.setenv("HEARTH_CUDA_SCOPE", "moe")
    with Engine(CUDA_LIB) as g:
        assert g.route_replay(trace) == 0
        got = session(g, other, 4)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
