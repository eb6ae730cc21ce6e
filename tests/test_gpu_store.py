"""The expert store's prefetch hints on the GPU (hx_store_prefetch, engine/src/hx_store.h:67-69 and
engine/src/store.c:435-580 of the reference): a hint whose expert is then routed counts as used, a
hint that is evicted unused counts as wasted, and a hint is dropped when the store has no cold,
unprotected slot for it. Results stay bit-identical to the oracle throughout."""
import numpy as np
import pytest

import hearth_b200 as hb
from tests.moe_util import backend_kwargs, bits, build_pair, load_weights, make_weights

pytestmark = pytest.mark.gpu

SLAB = 53248   # FORMAT §5 slab bytes of a Q4 expert at D 256, F 128


def _routing(kw, seed, hs):
    """Per token and layer the experts a resident handle routes to (same weights as build_pair(seed))."""
    layers = make_weights(seed, **kw)
    out = []
    with hb.MoeBackend(**backend_kwargs(**kw)) as be:
        load_weights(be, layers)
        for h in hs:
            ids = []
            x = h.copy()
            for l in range(kw["L"]):
                x = be.forward(x, layer0=l, n_layers=1)
                ids.append(set(int(e) for e in be.last_routing(h.shape[0])[0].reshape(-1)))
            out.append(ids)
    return out


def test_prefetch_hint_then_use_counts_as_used(gpu):
    kw = dict(L=2, E=16, K=4, max_tokens=1, cache_gb=18 * SLAB / 2**30, policy=1)
    h = np.random.default_rng(31).standard_normal((1, 256)).astype(np.float32)
    (ids0, _), = _routing(kw, 61, [h])
    model, be = build_pair(61, **kw)
    with be:
        assert be.stats()["n_slots"] == 18
        be.prefetch(0, sorted(ids0))
        st = be.stats()
        assert st["prefetch_issued"] == 4 and st["copies"] == 4
        got = be.forward(h, layer0=0, n_layers=1)
        st = be.stats()
        assert st["prefetch_used"] == 4 and st["prefetch_wasted"] == 0
        assert st["copies"] == 4   # the routed experts came from the hints, no demand copy
        assert np.array_equal(bits(got), bits(model.forward(h, n_layers=1)))


def test_prefetch_hint_evicted_unused_counts_as_wasted(gpu):
    kw = dict(L=2, E=32, K=2, max_tokens=1, cache_gb=34 * SLAB / 2**30, policy=1, prefetch_next=0)
    rng = np.random.default_rng(32)
    hs = [rng.standard_normal((1, 256)).astype(np.float32) for _ in range(30)]
    routed = _routing(kw, 62, hs)
    never = sorted(set(range(32)) - set().union(*(r[1] for r in routed)))
    assert never, "every layer-1 expert was routed: pick another seed"
    model, be = build_pair(62, **kw)
    with be:
        assert be.stats()["n_slots"] == 34
        be.prefetch(1, never)
        assert be.stats()["prefetch_issued"] == len(never)
        be.tick()
        be.tick()   # the hints' protection (until the next token) is over
        for h in hs:
            assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))
            be.tick()
        st = be.stats()
    assert st["evictions"] > 0
    assert st["prefetch_used"] == 0
    assert 1 <= st["prefetch_wasted"] <= len(never)


def test_prefetch_dropped_without_a_cold_slot(gpu):
    """LRU store whose every slot was used by the current token: a hint has no victim and is dropped;
    after the token boundary the least recently used slot becomes a victim and the hint is issued."""
    kw = dict(L=2, E=16, K=4, max_tokens=8, cache_gb=18 * SLAB / 2**30, policy=0, prefetch_next=0)
    h = np.random.default_rng(33).standard_normal((8, 256)).astype(np.float32)
    model, be = build_pair(63, **kw)
    with be:
        assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))
        st = be.stats()
        assert st["n_slots"] == 18 and st["evictions"] > 0   # more distinct experts than slots this token
        absent = [e for e in range(16) if not be.is_resident(1, e)]
        assert absent
        be.prefetch(1, absent[:1])
        assert be.stats()["prefetch_issued"] == 0           # dropped: every slot is hot this token
        be.tick()
        be.prefetch(1, absent[:1])
        assert be.stats()["prefetch_issued"] == 1
        assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))


@pytest.mark.parametrize("policy", [0, 1])
def test_next_layer_prediction_prefetches_while_a_layer_computes(gpu, policy):
    """With prefetch_next (the default) a streaming forward routes layer l+1 with layer l's input and
    hands the predicted experts to the store as hints (engine/src/model.c:944-973): hints are issued
    and used, results stay bit-identical to the oracle; with prefetch_next=0 no hint is issued."""
    L, E = 4, 16
    rng = np.random.default_rng(34)
    hs = [rng.standard_normal((1, 256)).astype(np.float32) for _ in range(6)]
    stats = {}
    for pn in (1, 0):
        model, be = build_pair(64, L=L, E=E, K=4, max_tokens=1, cache_gb=(E + 4) * SLAB / 2**30, policy=policy,
                               prefetch_next=pn)
        with be:
            assert be.stats()["n_slots"] < L * E
            for h in hs:
                assert np.array_equal(bits(be.forward(h)), bits(model.forward(h)))
                be.tick()
            stats[pn] = be.stats()
    assert stats[1]["prefetch_issued"] > 0 and stats[1]["prefetch_used"] > 0
    assert stats[1]["prefetch_used"] + stats[1]["prefetch_wasted"] <= stats[1]["prefetch_issued"]
    assert stats[0]["prefetch_issued"] == 0
