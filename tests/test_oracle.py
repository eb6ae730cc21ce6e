"""CPU checks of the oracle (the C restatement used as the checker) against the reference's own
golden vectors: its pinned FNV-1a hashes, its numpy routing and MoE code, its compiled kernels."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import oracle as O

# engine/tests/test_quant.c:56-62
PIN_Y = {0: 0x78ee7e5c72e238a0, 1: 0xacbfba9fb13b1207, 2: 0xaa0b6460cbd8ad23, 3: 0x532a2d32570c08dc,
         4: 0xa8a0369ab6f0ed22}
PIN_Q = {3: 0xda285a267ed1fb09, 4: 0x5ed717f72d36fb0c}


def test_det_fill_matches_fixture(golden):
    g = golden("pinned_matmul.npz")
    assert np.array_equal(O.det_fill(3 * 512, 2).reshape(3, 512), g["X"])


@pytest.mark.parametrize("dt", [0, 1, 2, 3, 4])
def test_oracle_reproduces_pinned_matmul_hashes(golden, dt):
    g = golden("pinned_matmul.npz")
    W, X = g[f"W{dt}"], g["X"]
    if dt in PIN_Q:
        assert O.fnv1a(W) == PIN_Q[dt]          # the fixture is the reference quantizer's output
    Y = O.matmul(dt, W, 24, 512, X)
    assert O.fnv1a(Y) == PIN_Y[dt]
    assert np.array_equal(Y.view(np.uint32), g[f"Y{dt}"].view(np.uint32))


def _route_cfg(cfg, rs):
    E, K, sf, sb, ng, tg, norm = [int(v) for v in cfg]
    return O.RouteCfg(E, K, sf, sb, ng, tg, norm, float(rs))


def test_oracle_routing_matches_numpy_reference(golden):
    g = golden("routing.npz")
    for name in g["cases"]:
        name = str(name)
        rc = _route_cfg(g[f"{name}__cfg"], g[f"{name}__rs"][0])
        logits, ids_ref, w_ref = g[f"{name}__logits"], g[f"{name}__ids"], g[f"{name}__w"]
        bias = g[f"{name}__bias"]
        E, K = rc.E, rc.K
        for t in range(logits.shape[0]):
            ids = np.zeros(K, np.int32)
            score = np.zeros(E, np.float32)
            w = np.zeros(K, np.float32)
            lg = np.ascontiguousarray(logits[t])
            O.lib().orc_route_select(C.byref(rc), lg.ctypes.data, bias.ctypes.data if bias.size else None, K,
                                     ids.ctypes.data, score.ctypes.data)
            O.lib().orc_route_weights(C.byref(rc), score.ctypes.data, ids.ctypes.data, w.ctypes.data)
            assert list(ids) == list(ids_ref[t]), (name, t)
            # numpy reference uses float64 exp rounded once; host expf agrees to <= 1 ulp
            np.testing.assert_array_max_ulp(w, w_ref[t], maxulp=2)


@pytest.mark.parametrize("name", ["qwen3_like", "deepseek_like", "qwen2_like"])
def test_oracle_moe_layer_matches_reference(golden, name):
    g = golden(f"moe_layer_{name}.npz")
    sf, sb, ng, tg, norm = [int(v) for v in g["cfg"]]
    D, F, E, K = int(g["D"]), int(g["F"]), int(g["E"]), int(g["K"])
    m = O.MoeModel(D, F, E, K, score_fn=sf, score_bias=sb, n_group=ng, topk_group=tg, norm_topk_prob=norm,
                   routed_scale=float(g["routed_scale"]))
    shared = None
    if int(g["Fs"]):
        shared = dict(Fs=int(g["Fs"]), dtype=O.Q8, gate=g["sh_gate"], up=g["sh_up"], down=g["sh_down"],
                      gate_inp=g["sh_gate_inp"] if g["sh_gate_inp"].size else None)
    m.add_layer(g["router"], list(g["slabs"]), [O.Q4] * E, bias=g["bias"] if g["bias"].size else None,
                shared=shared)
    y, ids, _ = m.layer_eval(0, g["x"])
    assert np.array_equal(ids, g["ids"])
    # bit-identical to the reference's compiled kernels (same host libm expf)
    assert np.array_equal(y.view(np.uint32), g["y_kernels"].view(np.uint32))
    # and to the numpy reference (float64 exp) within rounding
    np.testing.assert_allclose(y, g["y_numpy"], rtol=1e-5, atol=1e-7)


def test_route_union_orders_pairs():
    rng = np.random.default_rng(3)
    E, K, T = 16, 4, 9
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    ulist, u_p0, u_n = (np.zeros(E, np.int32) for _ in range(3))
    pair_tok, pair_of = np.zeros(T * K, np.int32), np.zeros(T * K, np.int32)
    nu = O.lib().orc_route_union(E, K, T, ids.ctypes.data, ulist.ctypes.data, u_p0.ctypes.data, u_n.ctypes.data,
                                 pair_tok.ctypes.data, pair_of.ctypes.data)
    assert list(ulist[:nu]) == sorted(set(ids.reshape(-1).tolist()))
    for u in range(nu):
        toks = pair_tok[u_p0[u]:u_p0[u] + u_n[u]]
        assert list(toks) == sorted(toks)
        for t in toks:
            assert ulist[u] in ids[t]
    for t in range(T):
        for j in range(K):
            p = pair_of[t * K + j]
            assert pair_tok[p] == t
            u = np.searchsorted(u_p0[:nu], p, side="right") - 1
            assert ulist[u] == ids[t, j]


def test_reference_kernels_equal_oracle_when_built():
    """The reference's own AVX-512 kernels (built from its sources) vs the oracle, T=3 Q4/Q8."""
    L = O.ref_lib()
    if L is None:
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(5)
    for dt in (3, 4):
        W = rng.standard_normal((40, 1024)).astype(np.float32)
        q = O.ref_quantize(dt, W, 2)
        X = rng.standard_normal((3, 1024)).astype(np.float32)
        Y = np.empty((3, 40), np.float32)
        assert L.hearth_matmul(dt, q.ctypes.data, 40, 1024, X.ctypes.data, 3, Y.ctypes.data, 0) == 0
        assert np.array_equal(Y.view(np.uint32), O.matmul(dt, q, 40, 1024, X).view(np.uint32))
