"""hxb_moe_load_container on the GPU: a handle opened from a .hearth file written by the reference's
own container writer (tests/golden/make_container.py) evaluates its MoE layers bit for bit like the
oracle on the same weights, with every expert resident and with a streaming store smaller than the
file's physical slabs; aliased entries read their target's slab."""
import numpy as np
import pytest

import hearth_b200 as hb
from tests.container_util import FIXTURE, FIXTURE_KW, fixture_layers
from tests.moe_util import bits, oracle_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cache_slabs", [0, 10])
@pytest.mark.parametrize("T", [1, 5])
def test_container_layers_equal_oracle(gpu, T, cache_slabs):
    model = oracle_model(fixture_layers(), **FIXTURE_KW)
    opts = dict(max_tokens=8)
    if cache_slabs:   # fewer slots than the 13 physical slabs (16 logical experts): streaming
        opts["cache_gb"] = cache_slabs * 16384 / 2**30
    be = hb.MoeBackend.from_container(FIXTURE, **opts)
    with be:
        if cache_slabs:
            assert be.stats()["n_slots"] < 13
        assert be.stats()["host_bytes"] == 13 * 16384   # 16 experts, 13 physical slabs: aliases share
        rng = np.random.default_rng(T)
        for _ in range(3):
            h = rng.standard_normal((T, 128)).astype(np.float32)
            got = be.forward(h, layer0=1, n_layers=2)   # layer 0 of the file is dense: not in the handle
            be.tick()
            assert np.array_equal(bits(got), bits(model.forward(h)))


@pytest.mark.parametrize("field,value", [("top_k", 3), ("norm_eps", 1e-5), ("residual_scale", 1.0),
                                         ("routed_scale", 2.5000002)])
def test_handle_that_disagrees_with_the_container_is_refused(gpu, field, value):
    """Every setting the kernels compute with must equal the container's (floats bit for bit): a
    handle with another epsilon or residual scale would give results the reference does not."""
    cfg, _ = hb.container_probe(FIXTURE)
    assert np.float32(cfg[field]) != np.float32(value)
    cfg[field] = value
    with hb.MoeBackend(**cfg, max_tokens=2) as be:
        with pytest.raises(RuntimeError, match="disagree"):
            be.load_container(FIXTURE)


@pytest.mark.parametrize("cache_slabs", [0, 10])
def test_setting_a_shared_slab_updates_its_aliases(gpu, cache_slabs):
    """(2, 6) is an alias of (1, 0): new bytes for (1, 0) reach both experts (their HBM copies are
    placed again in a resident handle, reloaded on demand in a streaming one)."""
    layers = fixture_layers()
    new = np.array(layers[1]["slabs"][3], copy=True)   # another expert's slab as the new bytes
    opts = dict(max_tokens=8, cache_gb=cache_slabs * 16384 / 2**30)
    with hb.MoeBackend.from_container(FIXTURE, **opts) as be:
        be.set_expert(1, 0, new)
        layers[0]["slabs"][0] = new
        layers[1]["slabs"][6] = new
        model = oracle_model(layers, **FIXTURE_KW)
        rng = np.random.default_rng(11)
        for _ in range(3):
            h = rng.standard_normal((6, 128)).astype(np.float32)
            got = be.forward(h, layer0=1, n_layers=2)
            be.tick()
            assert np.array_equal(bits(got), bits(model.forward(h)))


def test_new_bytes_for_a_shared_slab_during_a_prefetch_of_an_alias(gpu):
    """A prefetch copy of an alias (2, 6) reads the pinned buffer it shares with (1, 0); setting new
    bytes for (1, 0) while that copy may still be in flight waits for it first, so neither expert's
    HBM copy can mix old and new bytes: both then compute with the new slab."""
    layers = fixture_layers()
    new = np.array(layers[1]["slabs"][5], copy=True)
    with hb.MoeBackend.from_container(FIXTURE, max_tokens=8, cache_gb=10 * 16384 / 2**30) as be:
        for _ in range(4):
            be.prefetch(2, [6, 0, 1])   # layer index 2 of the handle = MoE layer 1 of the oracle list
            be.set_expert(1, 0, new)
        layers[0]["slabs"][0] = new
        layers[1]["slabs"][6] = new
        model = oracle_model(layers, **FIXTURE_KW)
        h = np.random.default_rng(12).standard_normal((4, 128)).astype(np.float32)
        assert np.array_equal(bits(be.forward(h, layer0=1, n_layers=2)), bits(model.forward(h)))
