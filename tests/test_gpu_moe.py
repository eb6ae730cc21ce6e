"""GPU parity of the MoE backend (router, Q4 experts, rank-order sum, shared expert, chained layers,
HBM expert store) against the oracle and the reference-derived golden fixtures. Bit-exact."""
import numpy as np
import pytest

import hearth_b200 as hb
from oracle import oracle as O
from tests.moe_util import bits, build_pair

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["qwen3_like", "deepseek_like", "qwen2_like"])
def test_layer_matches_reference_fixture(gpu, golden, name):
    g = golden(f"moe_layer_{name}.npz")
    sf, sb, ng, tg, norm = [int(v) for v in g["cfg"]]
    D, F, E, K, Fs = int(g["D"]), int(g["F"]), int(g["E"]), int(g["K"]), int(g["Fs"])
    gi = Fs and g["sh_gate_inp"].size > 0
    T = g["x"].shape[0]
    with hb.MoeBackend(n_layers=1, d_model=D, expert_ffn_dim=F, n_experts=E, top_k=K, score_fn=sf, score_bias=sb,
                       n_group=ng, topk_group=tg, norm_topk_prob=norm, routed_scale=float(g["routed_scale"]),
                       shared_ffn_dim=Fs, shared_dtype=O.Q8, shared_gate=int(bool(gi)), max_tokens=T) as be:
        be.set_layer(0, g["router"], g["bias"] if sb else None, None,
                     g["sh_gate"] if Fs else None, g["sh_up"] if Fs else None, g["sh_down"] if Fs else None,
                     g["sh_gate_inp"] if gi else None)
        for e in range(E):
            be.set_expert(0, e, g["slabs"][e])
        y = be.layer(0, g["x"])
        ids, _ = be.last_routing(T)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(bits(y), bits(g["y_kernels"]))


CASES = {
    "qwen3": dict(),
    "deepseek": dict(score_fn=1, score_bias=1, n_group=4, topk_group=2, routed_scale=2.5, Fs=128),
    "qwen2": dict(Fs=192, shared_gate=True, norm=0),
    "k1": dict(E=8, K=1),
}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("T", [1, 2, 7, 16, 17, 40])
def test_layer_equals_oracle(gpu, case, T):
    model, be = build_pair(100 + T, max_tokens=64, **CASES[case])
    with be:
        x = np.random.default_rng(T).standard_normal((T, 256)).astype(np.float32)
        y = be.layer(0, x)
        ids, w = be.last_routing(T)
    yo, ido, wo = model.layer_eval(0, x)
    assert np.array_equal(ids, ido)
    assert np.array_equal(bits(w), bits(wo))
    assert np.array_equal(bits(y), bits(yo))


@pytest.mark.parametrize("T", [1, 5, 24])
def test_forward_chain_equals_oracle(gpu, T):
    model, be = build_pair(7, L=3, max_tokens=32, residual_scale=0.5)
    with be:
        h = np.random.default_rng(1).standard_normal((T, 256)).astype(np.float32)
        hg = be.forward(h)
        hg2 = be.forward(h)          # replayed graph: same bits
    ho = model.forward(h)
    assert np.array_equal(bits(hg), bits(ho))
    assert np.array_equal(bits(hg2), bits(ho))


def test_batched_equals_sequential(gpu):
    """INV-DET-2: a batch gives every token exactly its single-token result."""
    model, be = build_pair(9, L=2, max_tokens=32)
    with be:
        h = np.random.default_rng(2).standard_normal((20, 256)).astype(np.float32)
        hb_ = be.forward(h)
        hs = np.stack([be.forward(h[i:i + 1])[0] for i in range(20)])
    assert np.array_equal(bits(hb_), bits(hs))


def test_streaming_store_equals_resident(gpu):
    """A cache smaller than the model: experts move host -> HBM on demand, with evictions;
    results identical to the all-resident run, and the counters add up."""
    L, E = 4, 16
    model, be_small = build_pair(21, L=L, E=E, max_tokens=8, cache_gb=(E + 4) * 53248 / 2**30, policy=1)
    with be_small:
        assert be_small.stats()["n_slots"] < L * E
        rng = np.random.default_rng(5)
        for step in range(6):
            h = rng.standard_normal((2, 256)).astype(np.float32)
            hg = be_small.forward(h)
            be_small.tick()
            assert np.array_equal(bits(hg), bits(model.forward(h)))
        st = be_small.stats()
        assert st["misses"] > 0 and st["evictions"] > 0
        assert st["hits"] + st["misses"] == st["expert_uses"] == 6 * 2 * 4 * L


def slab_nbytes(D, F):
    """FORMAT §5 slab size of a Q4 expert (gate, up at align64, down at align64, 4096-padded)."""
    rbd, rbf = D // 64 * 34, F // 64 * 34
    up = (F * rbd + 63) // 64 * 64
    down = (up + F * rbd + 63) // 64 * 64
    return (down + D * rbf + 4095) // 4096 * 4096


def test_streaming_store_staged_tensor_core(gpu):
    """Batches on the staged tensor-core kernels with a cache smaller than the model: each routed
    expert sits in whatever slot the store gave it (the tensor maps address the slab arena by slot),
    experts are evicted between layers, and the results equal the oracle."""
    L, E, D, F, T = 3, 16, 512, 256, 40
    model, be = build_pair(41, L=L, D=D, F=F, E=E, K=4, max_tokens=T,
                           cache_gb=(E + 4) * slab_nbytes(D, F) / 2**30)
    with be:
        assert be.stats()["n_slots"] < L * E
        rng = np.random.default_rng(9)
        for step in range(3):
            h = rng.standard_normal((T, D)).astype(np.float32)
            hg = be.forward(h)
            be.tick()
            assert np.array_equal(bits(hg), bits(model.forward(h)))
        assert be.stats()["evictions"] > 0


def test_lru_policy_streaming(gpu):
    L, E = 3, 16
    model, be = build_pair(22, L=L, E=E, max_tokens=4, cache_gb=(E + 2) * 53248 / 2**30, policy=0)
    with be:
        rng = np.random.default_rng(6)
        for _ in range(4):
            h = rng.standard_normal((1, 256)).astype(np.float32)
            assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))
            be.tick()


def test_copy_failure_returns_io_and_recovers(gpu):
    """Failure injection on the host side of the store: a failed copy makes the call return
    HX_E_IO (-4) without touching the caller's h; after the next tick the expert is read again."""
    L, E = 2, 16
    model, be = build_pair(23, L=L, E=E, max_tokens=4, cache_gb=(E + 2) * 53248 / 2**30)
    with be:
        fails = {"n": 0}

        def hook(layer, expert):
            if layer == 1 and fails["n"] < 1:
                fails["n"] += 1
                return 1
            return 0
        be.set_copy_hook(hook)
        h = np.random.default_rng(8).standard_normal((1, 256)).astype(np.float32)
        h0 = h.copy()
        with pytest.raises(RuntimeError, match="-4"):
            be.forward_into(h)
        assert np.array_equal(bits(h), bits(h0))
        assert be.stats()["copy_errors"] == 1
        be.tick()
        assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))


def test_capacity_and_argument_errors(gpu):
    model, be = build_pair(24, max_tokens=4)
    with be:
        with pytest.raises(RuntimeError, match="-3"):
            be.layer(0, np.zeros((5, 256), np.float32))
        with pytest.raises(RuntimeError, match="-1"):
            be.forward(np.zeros((1, 256), np.float32), layer0=1)


def test_heat_profile_pins(gpu):
    L, E = 2, 16
    model, be = build_pair(25, L=L, E=E, max_tokens=4, cache_gb=(E + 4) * 53248 / 2**30)
    with be:
        counts = np.zeros(L * E, np.float32)
        counts[[3, 17, 20]] = [5, 9, 7]
        be.seed_heat(counts, pin_fraction=0.15, warm_start=True)
        st = be.stats()
        assert st["pinned"] == 3
        assert be.is_resident(1, 1) and be.is_resident(0, 3) and be.is_resident(1, 4)
        h = np.random.default_rng(9).standard_normal((2, 256)).astype(np.float32)
        assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))


def _persistent_pair(seed, **kw):
    """Shapes the persistent decode kernels take (gate/up rows a multiple of 16 bytes)."""
    return build_pair(seed, **kw)


@pytest.mark.parametrize("case", ["softmax", "sigmoid_group", "nonorm", "sigmoid_bias"])
def test_persistent_decode_equals_oracle(gpu, case):
    kw = dict(L=3, D=512, F=256, E=32, K=4, max_tokens=4, residual_scale=0.7)
    if case == "sigmoid_group":
        kw.update(score_fn=1, score_bias=1, n_group=4, topk_group=2, routed_scale=2.5)
    if case == "nonorm":
        kw.update(norm=0, K=6)
    if case == "sigmoid_bias":
        kw.update(score_fn=1, score_bias=1, E=48, K=5, routed_scale=1.5)
    model, be = _persistent_pair(31, **kw)
    with be:
        assert be.decode_path() == "persistent"
        rng = np.random.default_rng(4)
        for _ in range(3):
            h = rng.standard_normal((1, 512)).astype(np.float32)
            hg = be.forward(h)
            assert np.array_equal(bits(hg), bits(model.forward(h)))
        ids, w = be.last_routing(1)
    assert ids.shape == (1, kw["K"])


@pytest.mark.parametrize("score_fn", [0, 1])
def test_persistent_decode_tied_scores(gpu, score_fn):
    """Duplicated router rows give bit-identical scores; the persistent kernel's selection breaks the
    ties by expert index exactly like the reference (lower index first), across its scoring warps."""
    E, K = 96, 8

    def tie(router):
        r = router.copy()
        for dst in (5, 40, 70, 95):      # a tie group spread over the four scoring warps, pushed up
            r[dst] = r[3]
        r[[3, 5, 40, 70, 95]] *= 4.0
        r[[12, 44]] = r[60]                # a second group, elsewhere in the order
        return r

    model, be = build_pair(51, L=2, D=512, F=256, E=E, K=K, score_fn=score_fn, max_tokens=1, router_fn=tie)
    rng = np.random.default_rng(8)
    with be:
        assert be.decode_path() == "persistent"
        for _ in range(4):
            h = rng.standard_normal((1, 512)).astype(np.float32)
            assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))
            ids, _ = be.last_routing(1)
            tied = [e for e in ids[0] if e in (3, 5, 40, 70, 95)]
            assert tied == sorted(tied)


@pytest.mark.parametrize("score_fn,nan_row", [(0, 0), (0, 9), (1, 7)])
def test_persistent_decode_nan_router_rows(gpu, score_fn, nan_row):
    """A NaN router row gives a NaN logit: with softmax every score turns NaN (the maximum keeps a
    leading NaN, the sum takes any NaN) and the selection falls back to expert order, NaN ranking
    last; with sigmoid only that expert's score is NaN and it is never selected. The warp routing's
    results equal the oracle's (NaN outputs compared as NaN)."""
    E, K = 32, 4

    def poison(router):
        r = router.copy()
        r[nan_row] = np.nan
        return r

    model, be = build_pair(53, L=2, D=512, F=256, E=E, K=K, score_fn=score_fn, max_tokens=1, router_fn=poison)
    rng = np.random.default_rng(9)
    with be:
        assert be.decode_path() == "persistent"
        for _ in range(2):
            h = rng.standard_normal((1, 512)).astype(np.float32)
            hg, hr = be.forward(h), model.forward(h)
            if score_fn == 0:
                assert np.isnan(hg).all() and np.isnan(hr).all()
                ids, _ = be.last_routing(1)
                assert list(ids[0]) == list(range(K))
            else:
                assert np.array_equal(bits(hg), bits(hr))
                ids, _ = be.last_routing(1)
                assert nan_row not in list(ids[0])


def test_persistent_decode_qwen3_shape_matches_multi_kernel_path(gpu, monkeypatch):
    """Qwen3-30B-A3B layer shape (D 2048, F 768, 128 experts, top-8), 2 layers: the persistent kernel,
    the multi-kernel path and the oracle agree bit for bit, and so does the last layer's routing."""
    model, be = build_pair(41, L=2, D=2048, F=768, E=128, K=8, max_tokens=1, router_sigma=0.02)
    rng = np.random.default_rng(5)
    hs = [rng.standard_normal((1, 2048)).astype(np.float32) for _ in range(3)]
    with be:
        assert be.decode_path() == "persistent"
        got = []
        for h in hs:
            got.append(be.forward(h))
            ids, w = be.last_routing(1)
        stats = be.stats()
    monkeypatch.setenv("HXB_PERSISTENT", "0")
    model2, be2 = build_pair(41, L=2, D=2048, F=768, E=128, K=8, max_tokens=1, router_sigma=0.02)
    with be2:
        assert be2.decode_path() == "layers"
        got2 = []
        for h in hs:
            got2.append(be2.forward(h))
            ids2, w2 = be2.last_routing(1)
    for h, a, b in zip(hs, got, got2):
        want = model.forward(h)
        assert np.array_equal(bits(a), bits(want))
        assert np.array_equal(bits(b), bits(want))
    assert np.array_equal(ids, ids2) and np.array_equal(bits(w), bits(w2))
    assert stats["expert_uses"] == 3 * 2 * 8


def test_persistent_decode_device_api_repeats(gpu):
    """forward_dev on a device buffer, many launches back to back (the barrier counter carries
    over between launches), then one sync."""
    import torch
    model, be = build_pair(43, L=2, D=512, F=256, E=32, K=4, max_tokens=1)
    with be:
        assert be.decode_path() == "persistent"
        rng = np.random.default_rng(6)
        h0 = rng.standard_normal((1, 512)).astype(np.float32)
        d = torch.from_numpy(h0.copy()).cuda()
        for _ in range(25):
            be.forward_dev(d, 1)
        be.sync()
        got = d.cpu().numpy()
    want = h0.copy()
    for _ in range(25):
        want = model.forward(want)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("T", [64, 100])
def test_tensor_core_stages_equal_oracle(gpu, case, T):
    """T * K >= 256 pairs: gate/up and down run on the tensor cores (tcgen05 .kind::i8, per-block int32
    tiles drained into the canonical float chains); the layer equals the oracle bit for bit."""
    kw = dict(CASES[case])
    if T * kw.get("K", 4) < 256:
        kw["K"] = 4
        T = 64
    model, be = build_pair(300 + T, max_tokens=T, **kw)
    with be:
        x = np.random.default_rng(T + 1).standard_normal((T, 256)).astype(np.float32)
        y = be.layer(0, x)
        ids, w = be.last_routing(T)
    yo, ido, wo = model.layer_eval(0, x)
    assert np.array_equal(ids, ido)
    assert np.array_equal(bits(w), bits(wo))
    assert np.array_equal(bits(y), bits(yo))


STAGED = {
    # D a multiple of 512 and Q4 experts: the persistent bulk-copy-staged tensor-core kernels
    "f256": dict(D=512, F=256, E=16, K=4, T=100),                    # down rows of 4 blocks, row pairs
    "f512_shared_q4": dict(D=512, F=512, E=16, K=8, T=70, Fs=512, shared_dtype=O.Q4, shared_gate=True),
    "f768_many_pair_tiles": dict(D=512, F=768, E=8, K=4, T=300),     # buckets of ~150 pairs: 5 pair tiles
    "sigmoid_groups": dict(D=1024, F=256, E=32, K=8, T=48, score_fn=1, score_bias=1, n_group=4, topk_group=2,
                           routed_scale=2.5, norm=0),
    "shared_f_differs": dict(D=512, F=256, E=16, K=4, T=80, Fs=384, shared_dtype=O.Q4),   # down: register path
}


@pytest.mark.parametrize("case", list(STAGED))
def test_staged_tensor_core_stages_equal_oracle(gpu, case):
    """Staged persistent tensor-core kernels (weight and activation rows brought into shared memory
    by bulk copies, a two-slot ring across tiles): routing, weights and outputs equal the oracle."""
    kw = dict(STAGED[case])
    T = kw.pop("T")
    model, be = build_pair(500 + T, max_tokens=T, **kw)
    with be:
        x = np.random.default_rng(T + 3).standard_normal((T, kw["D"])).astype(np.float32)
        y = be.layer(0, x)
        ids, w = be.last_routing(T)
    yo, ido, wo = model.layer_eval(0, x)
    assert np.array_equal(ids, ido)
    assert np.array_equal(bits(w), bits(wo))
    assert np.array_equal(bits(y), bits(yo))


def test_tensor_core_stages_qwen3_layer_shape(gpu):
    """The BASELINE single-layer shape (D 2048, F 768, 128 experts, top-8) with 40 tokens (320 pairs,
    six 128-row gate/up tiles, sixteen down tiles, partial token tiles) equals the oracle."""
    model, be = build_pair(331, L=1, D=2048, F=768, E=128, K=8, max_tokens=40, router_sigma=0.02)
    with be:
        x = np.random.default_rng(12).standard_normal((40, 2048)).astype(np.float32)
        y = be.layer(0, x)
    yo, _, _ = model.layer_eval(0, x)
    assert np.array_equal(bits(y), bits(yo))


@pytest.mark.parametrize("cache_gb", [0.0, 20 * 53248 / 2**30])
def test_forward_routed_with_the_computed_ids_equals_forward(gpu, cache_gb):
    """Route replay entry point: given exactly the ids the routing computes (layer by layer), the
    result equals the plain forward bit for bit; given other ids it differs (resident and streaming)."""
    L, T = 3, 4
    model, be = build_pair(71, L=L, E=16, K=4, max_tokens=T, cache_gb=cache_gb)
    with be:
        h = np.random.default_rng(13).standard_normal((T, 256)).astype(np.float32)
        ids, x = [], h.copy()
        for l in range(L):
            x = be.forward(x, layer0=l, n_layers=1)
            ids.append(be.last_routing(T)[0])
        ids = np.stack(ids)
        want = be.forward(h)
        assert np.array_equal(bits(be.forward_routed(h, ids)), bits(want))
        assert np.array_equal(bits(want), bits(model.forward(h)))
        other = (ids + 1) % 16
        assert not np.array_equal(bits(be.forward_routed(h, other)), bits(want))
        with pytest.raises(RuntimeError, match="-1"):
            be.forward_routed(h, np.full_like(ids, 16))
