"""Generates the whole-model fixtures tests/golden/tiny_<arch>.hearth with the REFERENCE's own tiny
model generator (python/hearth/synth.py make_tiny: random weights of each architecture's layout,
routers redrawn until every routing decision of its check sequence has a clear margin) and its
container writer, quantizing with the reference's C kernels compiled into oracle/_ref. Run here
(where the reference tree exists), never on the GPU box:

    python tests/golden/make_tiny_models.py [--ref <checkout of the reference repository>]

Fixtures (3 layers, d_model 128, 8 experts of width 64, top-2, vocab 256, max_seq 256):
  tiny_qwen3_moe.hearth  GQA 4/2 heads of 64 (head_dim != d_model / n_heads), per-head qk-norm,
                         RoPE theta 1e6, softmax top-k renormalised; Q4 experts, Q8 dense
  tiny_olmoe.hearth      MHA, full-width qk-norm, softmax without renormalisation; Q4 / Q8
  tiny_mixtral.hearth    GQA 4/2, no qk-norm; Q4 / Q8
  tiny_qwen2_moe.hearth  GQA 4/2, q/k/v biases, gated shared expert; Q8 experts and dense
  tiny_deepseek_v3.hearth  MLA attention (q-lora, kv-lora, GPT-J RoPE), a dense first layer, grouped
                         sigmoid routing with bias, shared expert; Q4 / Q8
  tiny_qwen3_moe_d512.hearth  the Qwen3 layout at d_model 512 (2 layers, 4 experts): rows of whole
                         16-byte units, so the single-token path takes the staged GEMVs with the fused
                         rmsnorm (q|k|v, LM head)
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

FIXTURES = [("qwen3_moe", "Q4", 11, {}), ("olmoe", "Q4", 12, {}), ("mixtral", "Q4", 13, {}),
            ("qwen2_moe", "Q8", 14, {}), ("deepseek_v3", "Q4", 15, {}),
            ("qwen3_moe", "Q4", 16, dict(n_layers=2, d_model=512, n_experts=4, top_k=2, expert_ffn=64))]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HEARTH_REF"),
                    help="the reference checkout (default: $HEARTH_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference checkout with --ref or HEARTH_REF")
    sys.path.insert(0, os.path.join(args.ref, "python"))
    os.environ.setdefault("HEARTH_LIB", os.path.join(REPO, "oracle", "_ref", "libhearth_ref.so"))
    from hearth import quant
    from hearth.synth import make_tiny
    for arch, dt, seed, shape in FIXTURES:
        name = f"tiny_{arch}" + (f"_d{shape['d_model']}" if shape else "")
        path = os.path.join(HERE, name + ".hearth")
        make_tiny(path, arch=arch, dtype=getattr(quant, dt), seed=seed, **shape)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
