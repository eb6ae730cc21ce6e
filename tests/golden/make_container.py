"""Generates tests/golden/tiny_moe.hearth (+ tiny_moe.npz) with the REFERENCE's own container writer
(python/hearth/format.py ContainerWriter, quantizing with the reference's C kernels built into
oracle/_ref), so that the container tests read a file the reference produced. Run here (where the
reference tree exists), never on the GPU box:

    python tests/golden/make_container.py [--ref <checkout of the reference repository>]

The container: 3 layers (layer 0 dense, layers 1 and 2 MoE), d_model 128, 8 Q4 experts of width 64,
top-2, sigmoid scores with a selection bias and 4 groups of which 2 are kept, normalised weights,
routed_scale 2.5, residual_scale 0.5, a Q8 shared expert of width 64 (ungated). Three expert entries
are aliases (flag bit 0): (2, 6) -> (1, 0), (2, 7) -> (1, 1), (2, 5) -> (2, 4). The MoE weights come
from tests/moe_util.make_weights (seed 77); every other canonical tensor is small random data.
tiny_moe.npz holds the MoE layers' router, bias, ffn_norm and shared-expert bytes for the oracle
(the expert slabs are read back from the container itself)."""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

D, F, E, K, FS, V, H, HD, FD = 128, 64, 8, 2, 64, 16, 2, 64, 64
ALIAS = {(2, 6): (1, 0), (2, 7): (1, 1), (2, 5): (2, 4)}
META = dict(arch="synthetic", n_layers=3, d_model=D, vocab_size=V, n_heads=H, n_kv_heads=H, head_dim=HD,
            layer_kind=[0, 1, 1], dense_ffn_dim=FD, n_experts=E, top_k=K, expert_ffn_dim=F, shared_ffn_dim=FS,
            shared_gate=0, score_fn=1, score_bias=1, n_group=4, topk_group=2, norm_topk_prob=1,
            routed_scale=2.5, residual_scale=0.5, norm_eps=1e-6, source="synthetic")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HEARTH_REF"),
                    help="the reference checkout (default: $HEARTH_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference checkout with --ref or HEARTH_REF")
    sys.path.insert(0, os.path.join(args.ref, "python"))
    sys.path.insert(0, REPO)
    # the reference's Python quantizer runs its own C kernels: oracle/_ref holds them, compiled from the
    # reference's sources by oracle/Makefile
    os.environ.setdefault("HEARTH_LIB", os.path.join(REPO, "oracle", "_ref", "libhearth_ref.so"))
    from hearth import quant
    from hearth.format import ContainerWriter, canonical_tensors, apply_defaults
    from tests.moe_util import make_weights

    layers = make_weights(77, L=2, D=D, F=F, E=E, Fs=FS, shared_gate=False, score_bias=1)
    rng = np.random.default_rng(5)
    path = os.path.join(HERE, "tiny_moe.hearth")
    c = apply_defaults(dict(META))
    tensors = canonical_tensors(c)
    moe_w = {1: layers[0], 2: layers[1]}
    with ContainerWriter(path, META) as w:
        for name, (shape, f32) in tensors.items():   # F32 where the format requires it
            w.declare_tensor(name, shape, quant.Q8 if ".shexp_" in name else (quant.F32 if f32 else quant.Q4))
        w.declare_experts(3, E, D, F, quant.Q4, [1, 2], alias=lambda l, e: ALIAS.get((l, e)))
        for name, (shape, f32) in tensors.items():
            l = int(name.split(".")[1]) if name.startswith("blk.") else -1
            lw = moe_w.get(l)
            if lw is not None and name.endswith(".moe_router"):
                w.write_tensor(name, lw["router"])
            elif lw is not None and name.endswith(".moe_router_bias"):
                w.write_tensor(name, lw["bias"])
            elif lw is not None and name.endswith(".ffn_norm"):
                w.write_tensor(name, lw["norm"])
            elif lw is not None and ".shexp_" in name:
                w.write_tensor(name, bytes(lw["shared"][name.split(".shexp_")[1]]))
            else:
                w.write_tensor(name, (rng.standard_normal(shape) * (0.02 if not f32 else 1.0)).astype(np.float32))
        rbd, rbf = D // 64 * 34, F // 64 * 34
        up = (F * rbd + 63) // 64 * 64
        down = (up + F * rbd + 63) // 64 * 64
        for l, lw in moe_w.items():
            for e in range(E):
                if (l, e) in ALIAS:
                    continue
                s = np.asarray(lw["slabs"][e], np.uint8)
                w.write_expert(l, e, bytes(s[:F * rbd]), bytes(s[up:up + F * rbd]), bytes(s[down:down + D * rbf]))
    np.savez_compressed(os.path.join(HERE, "tiny_moe.npz"),
                        router=np.stack([moe_w[l]["router"] for l in (1, 2)]),
                        bias=np.stack([moe_w[l]["bias"] for l in (1, 2)]),
                        norm=np.stack([moe_w[l]["norm"] for l in (1, 2)]),
                        sh_gate=np.stack([np.asarray(moe_w[l]["shared"]["gate"], np.uint8) for l in (1, 2)]),
                        sh_up=np.stack([np.asarray(moe_w[l]["shared"]["up"], np.uint8) for l in (1, 2)]),
                        sh_down=np.stack([np.asarray(moe_w[l]["shared"]["down"], np.uint8) for l in (1, 2)]))
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
