"""Generates the committed golden fixtures in tests/golden/ from the REFERENCE itself.

Run here (where the reference tree and its build exist), never on the GPU box:

    python tests/golden/make_golden.py [--ref <checkout of the reference repository>]

Sources of truth, all reference code:
* pinned_matmul.npz  — the reference's pinned-hash inputs (engine/tests/test_quant.c:873-887 det_fill,
  24x512 weights seed 1, 3x512 activations seed 2), quantized by the reference's own
  hearth_quantize, and the reference's hearth_matmul(isa=SCALAR) outputs for F32/F16/BF16/Q8/Q4.
* routing.npz        — router logits and the ids / weights chosen by the numpy reference's
  Reference._route (python/hearth/reference.py:432-463) for softmax and sigmoid-grouped configs,
  including exact ties.
* moe_layer_*.npz    — small MoE layers with reference-quantized Q4 experts (and a Q8 shared expert):
  inputs, the output of the numpy reference's Reference._moe (reference.py:465-479; float64 exp,
  so compared with a tolerance) and the output of the reference's compiled AVX-512 kernels driven
  by oracle/moe_ref.c (host libm expf, compared bit for bit).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402


def _stub_reference(Reference, cfg, E, K, D):
    """A Reference instance without a container: the routing / MoE code paths only."""
    r = object.__new__(Reference)
    r.cfg, r.E, r.K, r.D = cfg, E, K, D
    r._mats, r._vecs, r.router_trace, r._replay, r._moe_index = {}, {}, None, None, {0: 0}
    r.emulate = True
    return r


def pinned_matmul():
    R, C, TT = 24, 512, 3
    W = O.det_fill(R * C, 1).reshape(R, C)
    X = O.det_fill(TT * C, 2).reshape(TT, C)
    L = O.ref_lib()
    out = {"X": X}
    for dt in range(5):
        q = O.ref_quantize(dt, W, 3)
        Y = np.empty((TT, R), np.float32)
        rc = L.hearth_matmul(dt, q.ctypes.data, R, C, X.ctypes.data, TT, Y.ctypes.data, 1)
        assert rc == 0
        out[f"W{dt}"] = q
        out[f"Y{dt}"] = Y
    np.savez_compressed(os.path.join(HERE, "pinned_matmul.npz"), **out)


def routing(Reference, _Mat, quant):
    rng = np.random.default_rng(11)
    cases = []
    # (name, E, K, score_fn, score_bias, n_group, topk_group, norm, routed_scale)
    cfgs = [("softmax128_top8", 128, 8, 0, 0, 1, 1, 1, 1.0),
            ("softmax64_top8_nonorm", 64, 8, 0, 0, 1, 1, 0, 1.0),
            ("sigmoid256_group8_top8", 256, 8, 1, 1, 8, 4, 1, 2.5),
            ("sigmoid384_top8", 384, 8, 1, 1, 1, 1, 1, 2.827),
            ("softmax8_top2", 8, 2, 0, 0, 1, 1, 1, 1.0)]
    out = {}
    for name, E, K, sf, sb, ng, tg, norm, rs in cfgs:
        cfg = dict(score_fn=sf, score_bias=sb, n_group=ng, topk_group=tg, norm_topk_prob=norm, routed_scale=rs)
        D = 64
        n = 24
        logits = (rng.standard_normal((n, E)) * 2.0).astype(np.float32)
        logits[1, :] = 0.0                                   # all tied
        logits[2, 5] = logits[2, 3] = logits[2].max() + 1.0  # a tie at the top
        logits[3] = np.round(logits[3] * 2) / 2              # many ties
        bias = (rng.standard_normal(E) * 0.05).astype(np.float32) if sb else None
        if sb:
            bias[::7] = 0.0
        ids = np.zeros((n, K), np.int32)
        w = np.zeros((n, K), np.float32)
        for t in range(n):
            r = _stub_reference(Reference, cfg, E, K, D)
            # a matvec that returns the logits exactly: identity-like F32 router on a one-hot trick is
            # not needed — the stub matrix returns the prepared logits
            class _Logit:
                def __init__(self, v):
                    self.v = v

                def matvec(self, x):
                    return self.v.copy()
            r._mats["blk.0.moe_router#0"] = _Logit(logits[t])
            if bias is not None:
                r._vecs["blk.0.moe_router_bias"] = bias
            i_, w_ = Reference._route(r, 0, np.zeros(D, np.float32))
            ids[t], w[t] = i_, w_
        out[f"{name}__cfg"] = np.array([E, K, sf, sb, ng, tg, norm], np.int32)
        out[f"{name}__rs"] = np.array([rs], np.float32)
        out[f"{name}__logits"] = logits
        out[f"{name}__bias"] = bias if bias is not None else np.zeros(0, np.float32)
        out[f"{name}__ids"] = ids
        out[f"{name}__w"] = w
        cases.append(name)
    out["cases"] = np.array(cases)
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **out)


def moe_layers(Reference, _Mat, quant):
    specs = [
        # name, D, F, E, K, score_fn, score_bias, n_group, topk_group, norm, routed_scale, Fs, gate_inp, T, seed
        ("qwen3_like", 256, 128, 16, 4, 0, 0, 1, 1, 1, 1.0, 0, False, 6, 21),
        ("deepseek_like", 256, 128, 16, 4, 1, 1, 4, 2, 1, 2.5, 128, False, 5, 22),
        ("qwen2_like", 128, 64, 8, 2, 0, 0, 1, 1, 0, 1.0, 128, True, 4, 23),
    ]
    ref = O.MoeRef(n_threads=2)
    for name, D, F, E, K, sf, sb, ng, tg, norm, rs, Fs, gi, T, seed in specs:
        rng = np.random.default_rng(seed)
        router = (rng.standard_normal((E, D)) * 0.02 * 8).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.02).astype(np.float32) if sb else None
        up_off, down_off, nbytes = O.slab_layout(O.Q4, D, F)
        slabs = []
        for e in range(E):
            g = (rng.standard_normal((F, D)) * 0.02).astype(np.float32)
            u = (rng.standard_normal((F, D)) * 0.02).astype(np.float32)
            dn = (rng.standard_normal((D, F)) * 0.02).astype(np.float32)
            s = np.zeros(nbytes, np.uint8)
            qg, qu, qd = O.ref_quantize(O.Q4, g), O.ref_quantize(O.Q4, u), O.ref_quantize(O.Q4, dn)
            s[:qg.size] = qg.reshape(-1)
            s[up_off:up_off + qu.size] = qu.reshape(-1)
            s[down_off:down_off + qd.size] = qd.reshape(-1)
            slabs.append(s)
        shared = None
        if Fs:
            sg = O.ref_quantize(O.Q8, (rng.standard_normal((Fs, D)) * 0.02).astype(np.float32))
            su = O.ref_quantize(O.Q8, (rng.standard_normal((Fs, D)) * 0.02).astype(np.float32))
            sd = O.ref_quantize(O.Q8, (rng.standard_normal((D, Fs)) * 0.02).astype(np.float32))
            shared = dict(Fs=Fs, dtype=O.Q8, gate=sg, up=su, down=sd,
                          gate_inp=(rng.standard_normal(D) * 0.1).astype(np.float32) if gi else None)
        x = rng.standard_normal((T, D)).astype(np.float32)
        model = O.MoeModel(D, F, E, K, score_fn=sf, score_bias=sb, n_group=ng, topk_group=tg,
                           norm_topk_prob=norm, routed_scale=rs)
        model.add_layer(router, slabs, [O.Q4] * E, bias=bias, shared=shared)
        y_kern = ref.layer(model, 0, x)                      # reference kernels + libm expf
        y_orc, ids_orc, _ = model.layer_eval(0, x)
        assert np.array_equal(y_kern.view(np.uint32), y_orc.view(np.uint32)), name
        # the numpy reference's own MoE (float64 exp)
        cfg = dict(score_fn=sf, score_bias=sb, n_group=ng, topk_group=tg, norm_topk_prob=norm,
                   routed_scale=rs, shared_ffn_dim=Fs, shared_gate=1 if gi else 0)
        r = _stub_reference(Reference, cfg, E, K, D)
        r._mats["blk.0.moe_router#0"] = _Mat(quant.F32, E, D, w=router)
        if bias is not None:
            r._vecs["blk.0.moe_router_bias"] = bias
        mats = {}
        for e in range(E):
            s = slabs[e]
            mats[e] = (_Mat.from_bytes(s[:up_off].tobytes()[:F * O.row_bytes(O.Q4, D)], quant.Q4, F, D, True),
                       _Mat.from_bytes(s[up_off:up_off + F * O.row_bytes(O.Q4, D)].tobytes(), quant.Q4, F, D, True),
                       _Mat.from_bytes(s[down_off:down_off + D * O.row_bytes(O.Q4, F)].tobytes(), quant.Q4, D, F, True))
        r._expert = lambda layer, e: mats[e]
        if shared is not None:
            r._mats["blk.0.shexp_gate"] = _Mat.from_bytes(shared["gate"].tobytes(), quant.Q8, Fs, D, True)
            r._mats["blk.0.shexp_up"] = _Mat.from_bytes(shared["up"].tobytes(), quant.Q8, Fs, D, True)
            r._mats["blk.0.shexp_down"] = _Mat.from_bytes(shared["down"].tobytes(), quant.Q8, D, Fs, True)
            if gi:
                r._mats["blk.0.shexp_gate_inp#0"] = _Mat(quant.F32, 1, D, w=shared["gate_inp"].reshape(1, D))
        y_np = np.zeros((T, D), np.float32)
        ids_np = np.zeros((T, K), np.int32)
        for t in range(T):
            o, ids = Reference._moe(r, 0, x[t])
            y_np[t], ids_np[t] = o, ids
        assert np.array_equal(ids_np, ids_orc), name
        out = dict(D=D, F=F, E=E, K=K, cfg=np.array([sf, sb, ng, tg, norm], np.int32), routed_scale=np.float32(rs),
                   router=router, bias=bias if bias is not None else np.zeros(0, np.float32),
                   slabs=np.stack(slabs), x=x, y_kernels=y_kern, y_numpy=y_np, ids=ids_np, Fs=Fs)
        if shared is not None:
            out.update(sh_gate=shared["gate"], sh_up=shared["up"], sh_down=shared["down"],
                       sh_gate_inp=shared["gate_inp"] if gi else np.zeros(0, np.float32))
        np.savez_compressed(os.path.join(HERE, f"moe_layer_{name}.npz"), **out)
        print(name, "max |kernels - numpy| =", float(np.abs(y_kern - y_np).max()),
              "scale", float(np.abs(y_np).max()))
    ref.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HEARTH_REF"),
                    help="the reference checkout (default: $HEARTH_REF)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("name the reference checkout with --ref or HEARTH_REF")
    sys.path.insert(0, os.path.join(a.ref, "python"))
    from hearth.reference import Reference, _Mat  # noqa: E402
    from hearth import quant  # noqa: E402
    O.build()
    pinned_matmul()
    routing(Reference, _Mat, quant)
    moe_layers(Reference, _Mat, quant)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
