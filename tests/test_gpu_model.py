"""The whole decoder on the GPU (hxb_model_*) against the reference engine itself: the same container
and tokens evaluated by the reference's public API on the CPU (oracle/_ref/libhearth_ref.so,
hearth_eval) and by hearth_b200.Model give bit-identical logits for every prompt and decode
position, and the GPU's routing equals the rows of the reference's routing trace (docs/FORMAT.md §9
files written by hearth_trace_start). The containers are written by the reference's own tiny-model
generator and container writer (tests/golden/make_tiny_models.py, make_container.py): GQA with
per-head qk-norm (Qwen3), MHA with full-width qk-norm (OLMoE), GQA without qk-norm (Mixtral), q/k/v
biases and a gated Q8 shared expert (Qwen2-MoE), a dense first layer with a grouped sigmoid router
(tiny_moe), and the Qwen3 layout at d_model 512, whose single-token forwards take the staged GEMVs
with the rmsnorm formed inside them."""
import os

import numpy as np
import pytest

import hearth_b200 as hb
from tests.engine_util import REF_LIB, Engine, session

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MODELS = ["tiny_qwen3_moe", "tiny_olmoe", "tiny_mixtral", "tiny_qwen2_moe", "tiny_moe", "tiny_qwen3_moe_d512"]
PROMPT = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3]


def _path(name):
    return os.path.join(GOLDEN, name + ".hearth")


def _trace_rows(path):
    raw = open(path, "rb").read()
    hdr = np.frombuffer(raw[:24], np.uint32)   # magic, version, n_layers, n_experts, top_k, n_moe_layers
    assert hdr[0] == 0x52545248 and hdr[1] == 1
    w = int(hdr[5]) * int(hdr[4])
    return np.frombuffer(raw[24:], np.uint16).reshape(-1, w)


def _gpu_session(m, prompt, steps):
    rows = [m.eval(prompt, all_logits=True)]
    routes = [m.eval_routes()]
    tok = int(np.argmax(rows[0][-1]))
    for _ in range(steps):
        lg = m.eval([tok])
        routes.append(m.eval_routes())
        rows.append(lg[None, :])
        tok = int(np.argmax(lg))
    return np.concatenate(rows), np.concatenate(routes)


@pytest.mark.parametrize("name", MODELS)
def test_model_logits_and_routing_equal_the_reference_engines(gpu, name, tmp_path):
    trace = str(tmp_path / "cpu.trace")
    with Engine(REF_LIB, model=_path(name)) as cpu:
        want = session(cpu, PROMPT, 8, trace)
    with hb.Model(_path(name)) as m:
        got, routes = _gpu_session(m, PROMPT, 8)
    assert np.isfinite(want).all()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if m.n_moe:
        assert np.array_equal(routes, _trace_rows(trace))


@pytest.mark.parametrize("max_batch", [1, 5])
def test_prompt_in_chunks_equals_the_reference(gpu, max_batch):
    """The prompt split over several forward calls (max_batch), on both sides."""
    with Engine(REF_LIB, model=_path("tiny_qwen3_moe"), max_batch=max_batch) as cpu:
        want = session(cpu, PROMPT, 3)
    with hb.Model(_path("tiny_qwen3_moe"), max_batch=max_batch) as m:
        got, _ = _gpu_session(m, PROMPT, 3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_streaming_expert_store_gives_the_same_logits(gpu):
    """An HBM budget below the experts' bytes: the MoE layers stream their experts from pinned host
    memory (the store's minimum, E + 2 slots) with the same results."""
    with Engine(REF_LIB, model=_path("tiny_mixtral")) as cpu:
        want = session(cpu, PROMPT, 4)
    with hb.Model(_path("tiny_mixtral"), cache_gb=1e-4) as m:
        got, _ = _gpu_session(m, PROMPT, 4)
        st = m.moe_stats()
    assert st["n_slots"] < 3 * 8
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_route_replay_gives_the_reference_engines_logits(gpu, tmp_path):
    """hearth_route_replay: a trace recorded from another prompt drives the MoE layers of both."""
    name = "tiny_qwen3_moe"
    trace = str(tmp_path / "rec.trace")
    with Engine(REF_LIB, model=_path(name)) as rec:
        session(rec, PROMPT[::-1], 6, trace)
    other = [7, 2, 7, 1, 8, 2, 8, 1, 8, 2]
    with Engine(REF_LIB, model=_path(name)) as cpu:
        assert cpu.route_replay(trace) == 0
        want = session(cpu, other, 4)
    with hb.Model(_path(name)) as m:
        m.set_replay(_trace_rows(trace))
        got, routes = _gpu_session(m, other, 4)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    rows = _trace_rows(trace)
    assert np.array_equal(routes, rows[np.arange(len(other) + 4) % len(rows)])


def test_errors_leave_the_position(gpu):
    with hb.Model(_path("tiny_olmoe"), max_seq=20) as m:
        m.eval(PROMPT)
        assert m.pos == len(PROMPT)
        with pytest.raises(RuntimeError, match="-2"):
            m.eval([m.vocab])                  # HXB_E_TOKEN
        with pytest.raises(RuntimeError, match="-3"):
            m.eval(list(range(5)))             # beyond max_seq
        assert m.pos == len(PROMPT)
        m.eval([1, 2, 3, 4])                   # still usable
        assert m.pos == 20


def test_device_forward_equals_the_host_forward(gpu):
    """hxb_model_forward_dev (device ids and logits, asynchronous, single tokens replayed from a CUDA
    graph) gives the logits of hxb_model_forward."""
    import torch
    name = "tiny_qwen3_moe"
    with hb.Model(_path(name)) as a:
        want, _ = _gpu_session(a, PROMPT, 6)
    toks = [int(np.argmax(want[len(PROMPT) - 1]))] + [int(np.argmax(r)) for r in want[len(PROMPT):-1]]
    with hb.Model(_path(name)) as b:
        dev = torch.device("cuda", 0)
        lg = torch.empty((len(PROMPT), b.vocab), device=dev)
        b.forward_dev(torch.tensor(PROMPT, dtype=torch.int32, device=dev), 0, 2, lg)
        b.sync()
        rows = [lg.cpu().numpy()]
        one = torch.empty((1, b.vocab), device=dev)
        for i, t in enumerate(toks):
            b.forward_dev(torch.tensor([t], dtype=torch.int32, device=dev), len(PROMPT) + i, 1, one)
            b.sync()
            rows.append(one.cpu().numpy())
    got = np.concatenate(rows)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_synthesized_decoder_runs_and_repeats(gpu):
    """hxb_model_synthesize: a small all-MoE decoder generated in HBM; the same positions evaluated
    twice give the same logits (the KV cache rows are rewritten in place)."""
    with hb.Model.synthesize(vocab_size=512, n_heads=4, n_kv_heads=2, head_dim=64, qk_norm=1, n_layers=3,
                             d_model=256, expert_ffn_dim=128, n_experts=16, top_k=4, norm_topk_prob=1,
                             seed=3, max_batch=16, max_seq=64) as m:
        a = m.forward(np.arange(16, dtype=np.int32), 0, 2)
        b = [m.forward(np.array([7], np.int32), 16 + i, 1) for i in range(4)]
        a2 = m.forward(np.arange(16, dtype=np.int32), 0, 2)
        b2 = [m.forward(np.array([7], np.int32), 16 + i, 1) for i in range(4)]
    assert np.isfinite(a).all() and np.array_equal(a.view(np.uint32), a2.view(np.uint32))
    assert all(np.array_equal(x.view(np.uint32), y.view(np.uint32)) for x, y in zip(b, b2))
    assert not np.array_equal(b[0], b[1])   # positions differ
