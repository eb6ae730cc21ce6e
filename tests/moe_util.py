"""Shared helpers of the MoE tests: random layers with reference-quantized experts, loaded into
both the oracle model and the GPU backend."""
import numpy as np

import hearth_b200 as hb
from oracle import oracle as O


def q_matrix(rng, rows, cols, dt, sigma=0.02):
    W = (rng.standard_normal((rows, cols)) * sigma).astype(np.float32)
    if O.ref_lib() is not None:
        return O.ref_quantize(dt, W)
    # reference not built on this machine: synthetic valid blocks with realistic statistics
    bs = 34 if dt == O.Q4 else 66
    rb = O.row_bytes(dt, cols)
    q = np.zeros((rows, rb), np.uint8)
    nb = cols // 64
    for b in range(nb):
        blk = W[:, b * 64:(b + 1) * 64]
        amax = np.abs(blk).max(axis=1)
        if dt == O.Q4:
            d = (amax / 7.0).astype(np.float16)
            df = d.astype(np.float32)
            qi = np.clip(np.rint(blk / np.where(df == 0, 1, df)[:, None]), -8, 7).astype(np.int32) + 8
            q[:, b * bs:b * bs + 2] = d.view(np.uint8).reshape(rows, 2)
            q[:, b * bs + 2:b * bs + 34] = (qi[:, :32] | (qi[:, 32:] << 4)).astype(np.uint8)
        else:
            d = (amax / 127.0).astype(np.float16)
            df = d.astype(np.float32)
            qi = np.clip(np.rint(blk / np.where(df == 0, 1, df)[:, None]), -127, 127).astype(np.int8)
            q[:, b * bs:b * bs + 2] = d.view(np.uint8).reshape(rows, 2)
            q[:, b * bs + 2:b * bs + 66] = qi.view(np.uint8)
    return q


def make_slab(rng, D, F, dt=O.Q4):
    up, down, nb = O.slab_layout(dt, D, F)
    s = np.zeros(nb, np.uint8)
    g, u, d = q_matrix(rng, F, D, dt), q_matrix(rng, F, D, dt), q_matrix(rng, D, F, dt)
    s[:g.size] = g.reshape(-1)
    s[up:up + u.size] = u.reshape(-1)
    s[down:down + d.size] = d.reshape(-1)
    return s


def make_weights(seed, *, L=1, D=256, F=128, E=16, Fs=0, shared_gate=False, score_bias=0, router_sigma=0.15,
                 router_fn=None, shared_dtype=O.Q8, **_):
    """Random layer weights (reference-quantized experts) for L layers, reproducible from seed."""
    rng = np.random.default_rng(seed)
    layers = []
    for l in range(L):
        router = (rng.standard_normal((E, D)) * router_sigma).astype(np.float32)
        if router_fn is not None:
            router = np.ascontiguousarray(router_fn(router), np.float32)
        bias = (rng.standard_normal(E) * 0.05).astype(np.float32) if score_bias else None
        norm_w = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        slabs = [make_slab(rng, D, F) for _ in range(E)]
        shared = None
        if Fs:
            dt = shared_dtype
            shared = dict(Fs=Fs, dtype=dt, gate=q_matrix(rng, Fs, D, dt), up=q_matrix(rng, Fs, D, dt),
                          down=q_matrix(rng, D, Fs, dt),
                          gate_inp=(rng.standard_normal(D) * 0.1).astype(np.float32) if shared_gate else None)
        layers.append(dict(router=router, bias=bias, norm=norm_w, slabs=slabs, shared=shared))
    return layers


def load_weights(b, layers):
    """Loads make_weights' layers into a backend (an expert-parallel one keeps only its experts)."""
    for l, w in enumerate(layers):
        sh = w["shared"]
        b.set_layer(l, w["router"], w["bias"], w["norm"], sh["gate"] if sh else None, sh["up"] if sh else None,
                    sh["down"] if sh else None, sh["gate_inp"] if sh else None)
        for e, slab in enumerate(w["slabs"]):
            b.set_expert(l, e, slab)


def backend_kwargs(*, L=1, D=256, F=128, E=16, K=4, score_fn=0, score_bias=0, n_group=1, topk_group=1, norm=1,
                   routed_scale=1.0, Fs=0, shared_gate=False, max_tokens=64, cache_gb=0.0, policy=1,
                   residual_scale=1.0, shared_dtype=O.Q8, prefetch_next=1, **_):
    return dict(n_layers=L, d_model=D, expert_ffn_dim=F, n_experts=E, top_k=K, score_fn=score_fn,
                score_bias=score_bias, n_group=n_group, topk_group=topk_group, norm_topk_prob=norm,
                routed_scale=routed_scale, residual_scale=residual_scale, shared_ffn_dim=Fs,
                shared_dtype=shared_dtype, shared_gate=int(shared_gate), max_tokens=max_tokens, cache_gb=cache_gb,
                policy=policy, prefetch_next=prefetch_next)


def oracle_model(layers, *, D=256, F=128, E=16, K=4, score_fn=0, score_bias=0, n_group=1, topk_group=1, norm=1,
                 routed_scale=1.0, residual_scale=1.0, **_):
    model = O.MoeModel(D, F, E, K, score_fn=score_fn, score_bias=score_bias, n_group=n_group,
                       topk_group=topk_group, norm_topk_prob=norm, routed_scale=routed_scale,
                       residual_scale=residual_scale)
    for w in layers:
        model.add_layer(w["router"], w["slabs"], [O.Q4] * E, ffn_norm=w["norm"], bias=w["bias"], shared=w["shared"])
    return model


def build_pair(seed, *, ep_size=0, **kw):
    """An oracle model and a GPU backend holding the same random weights (make_weights' arguments;
    router_fn(router) may rewrite each layer's router matrix, e.g. duplicate rows to force tied
    scores). ep_size > 0 also opens ep_size expert-parallel handles (ranks 0..ep_size-1, same
    device) with the same weights and returns (model, backend, [handles])."""
    layers = make_weights(seed, **kw)
    model = oracle_model(layers, **kw)
    be = hb.MoeBackend(**backend_kwargs(**kw))
    load_weights(be, layers)
    eps = []
    for r in range(ep_size):
        eps.append(hb.MoeBackend(ep_size=ep_size, ep_rank=r, **backend_kwargs(**kw)))
        load_weights(eps[-1], layers)
    if ep_size:
        return model, be, eps
    return model, be


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)
