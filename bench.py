"""Benchmark: Q4 MoE decode through the Qwen3-30B-A3B-shaped MoE stack on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]
                    [--model qwen3|olmoe|mixtral|kimi] [--layers L]

Workload (one "step" = one decode step of B tokens through the hot path of every layer):
48 MoE layers of Qwen3-30B-A3B shape — per layer x = rmsnorm(h, ffn_norm), router [128 x 2048]
f32, softmax top-8 renormalised, 8 Q4 experts (gate/up 2048->768, down 768->2048, SwiGLU), the
rank-order expert sum and h += sum. Attention and the LM head are not on this path (they are the
reference's dense backbone, outside the MoE hot path), so tok/s counts the MoE stack only.
Weights are synthetic (seeded, N(0, 0.02)-like Q4 statistics), generated in HBM; every expert is
resident (14.7 GB). N > 1 (torchrun): the same token stream through the stack with the experts spread
over the ranks (expert e on rank e % N), strong scaling: at batch 1 one persistent kernel per token
and rank, the owners storing their experts' outputs into every GPU's memory over NVLink; --replicas
instead runs N independent replicas (weak scaling, no exchange).
--model selects another configuration's MoE stack (OLMoE-1B-7B, Mixtral-8x7B at batch 8, Kimi-K2
with its grouped sigmoid router, selection bias and Q8 shared expert), same line format.

value  : tokens/s with inputs resident in HBM (CUDA events on the launching stream, max over ranks)
e2e    : tokens/s through the public C ABI with host buffers (hxb_moe_forward: pinned-host copies
         of h in and out every step, inside the timed region)
--impl reference: the reference's own AVX-512 kernels + thread pool (oracle/_ref, built from the
         reference sources) on all host cores, same workload and byte-identical weights.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "Q4 MoE decode tok/s (Qwen3-30B-A3B shape); expert-GEMV HBM GB/s vs peak"
SIGMA = 0.02

# The MoE stacks of the benchmark configurations (routing as each architecture defines it; the
# seed is the configuration's). qwen3 is the headline workload; the others are --model modes.
MODELS = {
    "qwen3": dict(name="qwen3-30b-a3b", layers=48, D=2048, F=768, E=128, K=8, seed=2, batch=1,
                  route=dict(score_fn=0, norm_topk_prob=1),
                  dense=dict(vocab_size=151936, n_heads=32, n_kv_heads=4, head_dim=128, qk_norm=1, rope_theta=1e6)),
    "olmoe": dict(name="olmoe-1b-7b", layers=16, D=2048, F=1024, E=64, K=8, seed=1, batch=1,
                  route=dict(score_fn=0, norm_topk_prob=0),
                  dense=dict(vocab_size=50304, n_heads=16, n_kv_heads=16, head_dim=128, qk_norm=2, rope_theta=1e4)),
    "mixtral": dict(name="mixtral-8x7b", layers=32, D=4096, F=14336, E=8, K=2, seed=3, batch=8,
                    route=dict(score_fn=0, norm_topk_prob=1),
                    dense=dict(vocab_size=32000, n_heads=32, n_kv_heads=8, head_dim=128, qk_norm=0, rope_theta=1e6)),
    # Kimi-K2 / DeepSeek-V3: 60 MoE layers (the first of 61 is dense), sigmoid scores + selection
    # bias, 8 groups keep 4, routed_scale 2.827, one Q8 shared expert of width 2048
    "kimi": dict(name="kimi-k2", layers=60, D=7168, F=2048, E=384, K=8, seed=4, batch=1, Fs=2048,
                 route=dict(score_fn=1, score_bias=1, n_group=8, topk_group=4, norm_topk_prob=1,
                            routed_scale=2.827)),
}
MODEL = "qwen3"
L_, D_, F_, E_, K_ = 48, 2048, 768, 128, 8
FS_ = 0
SEED = 2


def set_model(key, layers=None, world=1):
    """Selects the stack; layers default to the model's, or to as many as fit the GPUs' HBM (~150 GB
    of expert slabs per GPU) when the whole stack does not."""
    global MODEL, L_, D_, F_, E_, K_, FS_, SEED
    m = MODELS[key]
    MODEL, D_, F_, E_, K_, FS_, SEED = key, m["D"], m["F"], m["E"], m["K"], m.get("Fs", 0), m["seed"]
    per_layer = E_ * slab_bytes()
    fit = max(1, int(world * 150e9 // per_layer))
    L_ = layers or min(m["layers"], fit)


def slab_bytes():
    """FORMAT §5 slab of one Q4 expert: gate/up [F, D] and down [D, F] at 64-byte aligned offsets,
    padded to 4096."""
    a = lambda n, k: (n + k - 1) // k * k
    g = F_ * (34 * D_ // 64)
    return a(a(a(g, 64) + g, 64) + D_ * (34 * F_ // 64), 4096)


def backend_kw(**extra):
    """MoeBackend arguments of the selected stack."""
    m = MODELS[MODEL]
    kw = dict(n_layers=L_, d_model=D_, expert_ffn_dim=F_, n_experts=E_, top_k=K_, shared_ffn_dim=FS_,
              shared_dtype=3, **m["route"])
    kw.update(extra)
    return kw


def batch_gateup_bytes(B):
    """Algorithmic bytes of one launch of the staged tensor-core gate/up kernel at batch B: the gate and
    up rows of every expert the batch routes to, read once (expected distinct experts of B tokens
    drawing K of E), the B activation rows read once and the B * K mid rows written once."""
    q4_row_d = 34 * D_ // 64
    experts = E_ * (1.0 - (1.0 - K_ / E_) ** B)
    return round(experts * 2 * F_ * q4_row_d + B * (D_ // 64) * 72 + B * K_ * (F_ // 64) * 72)


def algorithmic_bytes():
    """Bytes the path must read per token and layer (B = 1), FORMAT §6 row sizes: K experts' gate,
    up and down rows, the router (and selection bias), the norm, and a shared expert's Q8 rows."""
    q4_row_d = 34 * D_ // 64            # gate/up row (Qwen3: 1088 B)
    q4_row_f = 34 * F_ // 64            # down row (Qwen3: 408 B)
    expert = 2 * F_ * q4_row_d + D_ * q4_row_f
    router = E_ * D_ * 4 + (E_ * 4 if MODELS[MODEL]["route"].get("score_bias") else 0)
    shared = 2 * FS_ * (66 * D_ // 64) + D_ * (66 * FS_ // 64) if FS_ else 0
    return dict(gateup=K_ * 2 * F_ * q4_row_d, down=K_ * D_ * q4_row_f, router=router, norm=D_ * 4,
                shared=shared, layer=K_ * expert + router + D_ * 4 + shared, expert=expert)


def step_bytes(B):
    """Algorithmic bytes of one step of B tokens through the stack: per layer the expected distinct
    experts of B tokens drawing K of E (all K at B = 1), the router, the norm and the shared expert."""
    ab = algorithmic_bytes()
    experts = K_ if B == 1 else E_ * (1.0 - (1.0 - K_ / E_) ** B)
    return round(L_ * (experts * ab["expert"] + ab["router"] + ab["norm"] + ab["shared"]))


# DRAM bytes (read + write) per layer of k_moe_decode from one ncu capture of a 4-layer launch of the
# same shape (bench.py --layers 4: dram__bytes_read.sum 84.71 MB, dram__bytes_write.sum 2.30 MB); a
# launch's traffic grows with its layers, so the full launch's figure is this times its layers.
DECODE_DRAM_BYTES_PER_LAYER = (84_705_536 + 2_298_624) / 4


def workload_config(B, world, parallelism=None):
    """The line's config (identical in both arms: the reference arm times the same workload)."""
    m = MODELS[MODEL]
    cfg = {"workload": f"{m['name']} MoE stack {'decode' if B == 1 else 'batch step'}, {L_} layers, batch {B}",
           "layers": L_, "d_model": D_, "expert_ffn_dim": F_, "n_experts": E_, "top_k": K_, "batch": B,
           "parallelism": parallelism or f"replica x{world}",
           "l2": f"no flush: each step reads ~{L_ * algorithmic_bytes()['layer'] / 1e9:.2f} GB of expert/router "
                 "weights (> 126 MB L2)",
           "weights": "synthetic: seeded Q4 blocks with the statistics of N(0, 0.02) weights packed to Q4 and "
                      "an N(0, 0.02) f32 router, generated by the library's device generator (the CPU arm "
                      "generates the same bytes on the host)"}
    if MODEL != "qwen3":
        cfg["routing"] = dict(m["route"])
        if FS_:
            cfg["shared_expert"] = {"ffn_dim": FS_, "dtype": "q8"}
        if L_ < m["layers"]:
            cfg["layers_note"] = f"{L_} of the model's {m['layers']} MoE layers: as many as fit the GPUs' HBM"
    return cfg


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def max_over_ranks(v: float, world: int, device=None) -> float:
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_model(ref, n_layers):
    """The benchmark's model on the host, byte-identical to hxb_moe_synthesize(SEED): the router, the
    selection bias and the shared expert of layer l from seed SEED * 1000003 + l, the slabs from SEED."""
    from oracle import oracle as O
    up, down, nb = O.slab_layout(O.Q4, D_, F_)
    slabs = ref.synth_q4(n_layers * E_, nb, D_, F_, SEED, SIGMA)
    route = MODELS[MODEL]["route"]
    model = O.MoeModel(D_, F_, E_, K_, eps=1e-6, residual_scale=1.0, **route)
    for l in range(n_layers):
        ls = SEED * 1000003 + l
        router = ref.synth_f32(E_ * D_, ls, SIGMA).reshape(E_, D_)
        bias = ref.synth_f32(E_, ls ^ 0xb1a5b1a5, 0.5 * SIGMA) if route.get("score_bias") else None
        shared = None
        if FS_:
            shared = dict(Fs=FS_, dtype=O.Q8, gate=ref.synth_blocks(O.Q8, FS_, D_, ls ^ 0x5a1, SIGMA),
                          up=ref.synth_blocks(O.Q8, FS_, D_, ls ^ 0x5a2, SIGMA),
                          down=ref.synth_blocks(O.Q8, D_, FS_, ls ^ 0x5a3, SIGMA), gate_inp=None)
        model.add_layer(router, [slabs[l * E_ + e] for e in range(E_)], [O.Q4] * E_, bias=bias, shared=shared)
    return model, slabs


def time_cpu(ref, model, arr, B, tokens_budget_s: float, max_tokens: int, rng):
    """Times decode steps of B tokens on the host; returns (tokens/s, tokens timed, outputs, inputs)."""
    h0 = rng.standard_normal((B, D_)).astype(np.float32)
    ref.forward(model, h0.copy(), arr)                       # warm pass
    ins, outs = [], []
    t0 = time.perf_counter()
    n = 0
    while n < max_tokens:
        h = rng.standard_normal((B, D_)).astype(np.float32)
        ins.append(h.copy())
        ref.forward(model, h, arr)
        outs.append(h)
        n += 1
        if time.perf_counter() - t0 > tokens_budget_s:
            break
    dt = time.perf_counter() - t0
    return n * B / dt, n, ins, outs


def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path (rank 0 only)."""
    if rank != 0:
        return
    from oracle import oracle as O
    if O.moe_ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference sources absent)"}))
        return
    if MODEL == "kimi":
        print(json.dumps({"impl": "reference", "unavailable": "the Kimi-K2 stack's experts (539 GB) exceed the "
                                                              "host memory the CPU arm would hold them in"}))
        return
    ref = O.MoeRef(n_threads=0)
    model, _ = cpu_model(ref, L_)
    arr = model.c_layers()
    rng = np.random.default_rng(123)
    for _ in range(max(1, min(args.warmup, 3))):
        ref.forward(model, rng.standard_normal((args.batch, D_)).astype(np.float32), arr)
    # bounded sample: at most ~60 s of timed work whatever --steps says
    tps, n, _, _ = time_cpu(ref, model, arr, args.batch, 60.0, args.steps, rng)
    line = {"metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "ms_per_step": round(1000.0 * args.batch / tps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4xq8-int32+f32", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(args.batch, args.gpus),
            "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": ref.threads, "kind": "reference",
                             "sample": f"{n} decode steps of batch {args.batch} (60 s cap), reference AVX-512 "
                                       f"kernels (isa {ref.isa}) + hx_pool on {ref.threads} threads"},
            "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    ref.close()


TRACE_STAMPS = ["start", "h polled", "rmsnorm chain", "router rows in", "x", "logit stored", "activation blocks",
                "logits polled", "routed",
                "routing barrier", "first chunk landed", "its SwiGLU stored", "exchange reset", "mid polled", "mid blocks",
                "down rows landed", "down rows computed", "y stored", "y polled", "h stored"]


def run_trace(args, local_rank):
    """Per-phase timeline of the persistent decode kernel (one JSON line): for each stamp, the mean and
    the per-layer maximum over CTAs of the interval from the previous stamp, in us at the SM clock."""
    os.environ["HXB_TRACE"] = "1"
    import torch
    import hearth_b200 as hb
    torch.cuda.set_device(local_rank)
    be = hb.MoeBackend(**backend_kw(max_tokens=1, device=local_rank))
    be.synthesize(SEED, SIGMA, SIGMA)
    g = torch.Generator(device="cuda").manual_seed(1000)
    pool = torch.randn((64, 1, D_), generator=g, device="cuda")
    s = torch.cuda.current_stream()
    for i in range(max(args.warmup, 3)):
        be.forward_dev(pool[i % 64], 1, stream=s)
    be.sync(s)
    # stamps are SM clock cycles: convert at the median SM clock sampled while the traced launches run
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    for i in range(2000):
        be.forward_dev(pool[i % 64], 1, stream=s)
    be.sync(s)
    clk = clocks.stop()
    t = be.phase_trace()
    S = len(TRACE_STAMPS)
    t = t.reshape(L_, -1, S).astype(np.int64)
    mhz = clk["sm_mhz"] or clk["sm_max_mhz"]
    if not mhz:
        raise RuntimeError("no SM clock samples: the trace cannot be converted to time")
    d = np.diff(t, axis=2) / mhz
    phases = {TRACE_STAMPS[i + 1]: {"mean_us": round(float(d[:, :, i].mean()), 3),
                                    "max_us": round(float(d[:, :, i].max(axis=1).mean()), 3)} for i in range(S - 1)}
    layer = (t[:, :, S - 1] - t[:, :, 0]) / mhz
    print(json.dumps({"trace": "k_moe_decode phases", "layers": L_, "ctas": int(t.shape[1]), "clock_mhz": mhz,
                      "clock": "median SM MHz sampled during the traced launches", "clocks": clk,
                      "layer_us_mean": round(float(layer.mean()), 3), "phases": phases}), flush=True)


def run_ep(args, rank, world, local_rank):
    """One token stream through the MoE stack with the experts spread over the ranks (expert e on rank
    e % world): per layer every rank routes the batch, computes its experts' pairs, the ranks all-gather
    the pairs' outputs (NCCL) and each forms the rank-order sum. Total work is fixed as N grows."""
    import torch
    import torch.distributed as dist
    import hearth_b200 as hb
    from hearth_b200.ep import ExpertParallelMoe
    dev = torch.device("cuda", local_rank)
    B = args.batch
    be = hb.MoeBackend(**backend_kw(max_tokens=B, device=local_rank, ep_size=world, ep_rank=rank))
    be.synthesize(SEED, SIGMA, SIGMA)
    ep = ExpertParallelMoe(be)
    dist.barrier()
    P = 64
    g = torch.Generator(device=dev).manual_seed(1000)   # the same tokens on every rank
    pool = torch.randn((P, B, D_), generator=g, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    for i in range(max(args.warmup, 3)):
        ep.forward_dev(pool[i % P], B, stream=stream)
    be.sync(stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        ep.forward_dev(pool[i % P], B, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    be.sync(stream)
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    dist.barrier()
    clk = clocks.stop()
    value = args.steps * B / (ms / 1000.0)
    # end to end: the token from pinned host memory and back each step
    hin = torch.randn((B, D_), generator=torch.Generator().manual_seed(7)).pin_memory()
    hout = torch.empty_like(hin).pin_memory()
    hd = torch.empty((B, D_), device=dev)
    n_e2e = min(args.steps, 500)
    torch.cuda.synchronize(dev)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        hd.copy_(hin, non_blocking=True)
        ep.forward_dev(hd, B, stream=stream)
        hout.copy_(hd, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    t_e2e = max_over_ranks(time.perf_counter() - t0, world, dev)
    ab = algorithmic_bytes()
    hbm, peak_kind = peaks()
    gbs = step_bytes(B) / (ms / args.steps * 1e-3) / 1e9   # whole-stack bytes over all ranks
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "q4xq8-int32+f32", "data": "synthetic",
                "config": workload_config(B, world, f"ep{world}"),
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": round(hbm * world, 1), "unit": "GB/s",
                             "frac": round(gbs / (hbm * world), 4), "traffic": None,
                             "kernel": ("k_moe_decode expert-parallel (one launch per token and rank; y rows stored "
                                        "into every GPU over NVLink)" if ep.connected and B == 1 else
                                        "per-phase kernels + NCCL all-gather per layer"),
                             "peak_kind": peak_kind},
                "cpu_baseline": None,
                "e2e": {"value": round(n_e2e * B / t_e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": B * D_ * 4,
                        "d2h_bytes_per_step": B * D_ * 4, "timing": "host clock, pinned copies in and out per step"},
                "gpu_launches": args.steps * (1 if ep.connected and B == 1 else L_ * 7), "clocks": clk}
        print(json.dumps(line), flush=True)
    be.close()


def full_bytes_per_token(pos):
    """Algorithmic bytes of one decode token through the whole decoder at position pos: the MoE
    stack's (step_bytes(1)), the attention projections and the LM head in Q8 (FORMAT §6 rows), the
    embedding row, the norms, and the KV rows read (f32 k and v of positions 0..pos) and written."""
    d = MODELS[MODEL]["dense"]
    q8 = lambda n: 66 * n // 64
    qd, kvd = d["n_heads"] * d["head_dim"], d["n_kv_heads"] * d["head_dim"]
    attn = (qd + 2 * kvd) * q8(D_) + D_ * q8(qd) + 4 * D_
    head = d["vocab_size"] * q8(D_) + 4 * D_
    kv = 2 * kvd * 4 * (pos + 1)
    return dict(moe=step_bytes(1), attn=L_ * attn, head=head + q8(D_), kv=L_ * kv,
                total=step_bytes(1) + L_ * (attn + kv) + head + q8(D_))


def run_full(args, rank, world, local_rank):
    """The whole decoder (configuration 3 of the benchmark: a 512-token prompt, then decode steps at
    batch 1): embedding, 48 layers of GQA attention with the KV cache and the MoE stack, LM head,
    all on one GPU (hxb_model_synthesize weights). One step = one decode token at positions
    512..1023 (cycling), its logits written to HBM; e2e = the same through hxb_model_forward with host
    ids and logits."""
    import torch
    import hearth_b200 as hb
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    d = MODELS[MODEL]["dense"]
    P0, SEQ = 512, 1024
    m = hb.Model.synthesize(seed=SEED, device=local_rank, max_batch=P0, max_seq=SEQ, **d, **backend_kw())
    V = d["vocab_size"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    prompt = torch.randint(0, V, (P0,), generator=g, device=dev, dtype=torch.int32)
    pool = torch.randint(0, V, (64, 1), generator=g, device=dev, dtype=torch.int32)
    logits = torch.empty((1, V), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    # prefill, timed once after a warm pass
    m.forward_dev(prompt, 0, 0, stream=stream)
    m.sync(stream)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    m.forward_dev(prompt, 0, 0, stream=stream)
    p1.record(stream)
    m.sync(stream)
    prefill_ms = p0.elapsed_time(p1)
    for i in range(max(args.warmup, 3)):
        m.forward_dev(pool[i % 64], P0 + i % (SEQ - P0), 1, logits, stream=stream)
    m.sync(stream)
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        m.forward_dev(pool[i % 64], P0 + i % (SEQ - P0), 1, logits, stream=stream)
    e1.record(stream)
    m.sync(stream)
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    value = args.steps / (ms / 1000.0)
    assert torch.isfinite(logits).all().item()
    # end to end: host ids in, host logits out, every step
    n_e2e = min(args.steps, 1000)
    host_tok = np.random.default_rng(7).integers(0, V, size=64).astype(np.int32)
    out = np.empty(V, np.float32)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        out = m.forward(host_tok[i % 64:i % 64 + 1], P0 + i % (SEQ - P0), 1)
    t_e2e = time.perf_counter() - t0
    hbm, peak_kind = peaks()
    npos = min(args.steps, SEQ - P0)
    mean_pos = P0 + (npos - 1) / 2.0
    fb = full_bytes_per_token(int(mean_pos))
    gbs = fb["total"] / (ms / args.steps * 1e-3) / 1e9
    # embedding; per layer rmsnorm(+act), q|k|v, post, scores, softmax+values(+act), o(+residual) and
    # the MoE layer (one persistent launch, or four per-phase kernels); norm, LM head, scale, position
    moe_launches = 1 if hb.lib().hxb_moe_decode_path(hb.lib().hxb_model_moe(m.h)) == 1 else 4
    launches = 1 + L_ * (6 + moe_launches) + 4
    line = {"metric": "Q4 MoE decode tok/s, whole decoder (Qwen3-30B-A3B shape); HBM GB/s of expert+dense+KV bytes",
            "value": round(value, 3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4/q8xq8-int32+f32", "data": "synthetic",
            "config": {"workload": f"{MODELS[MODEL]['name']} whole decoder: {P0}-token prompt, then decode steps at "
                                   f"positions {P0}..{SEQ - 1} (cycling), batch 1",
                       "layers": L_, "d_model": D_, "n_heads": d["n_heads"], "n_kv_heads": d["n_kv_heads"],
                       "head_dim": d["head_dim"], "vocab": V, "experts": E_, "top_k": K_, "expert_ffn_dim": F_,
                       "parallelism": "single GPU",
                       "l2": f"no flush: each step reads ~{fb['total'] / 1e9:.2f} GB (> 126 MB L2)",
                       "weights": "synthetic: the library's device generator (Q8 dense, Q4 experts, f32 routers)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "traffic": None, "peak_kind": peak_kind,
                         "kernel": "the whole decode step (one CUDA graph: embedding, attention, MoE, LM head)",
                         "bytes_per_step": fb, "mean_position": mean_pos},
            "prefill": {"tokens": P0, "ms": round(prefill_ms, 3), "tok_s": round(P0 / prefill_ms * 1000.0, 1)},
            "cpu_baseline": None,
            "cpu_baseline_note": "the reference engine needs a container of this model (17 GB) that is not written "
                                 "on the GPU box; its CPU decode of the MoE stack is the headline line's baseline",
            "e2e": {"value": round(n_e2e / t_e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * V, "timing": "host clock around synchronous hxb_model_forward"},
            "gpu_launches": launches * args.steps, "clocks": clk}
    print(json.dumps(line), flush=True)
    m.close()


def run_stream(args, rank, world, local_rank):
    """The MoE stack with an HBM budget below its experts' bytes (--cache-gb): the experts live in the
    store's pinned host tier and stream into HBM slots per layer (routing read back, demand copies,
    next-layer prediction as prefetch hints), the hxb_moe path a container larger than HBM takes."""
    import torch
    import hearth_b200 as hb
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B = args.batch
    be = hb.MoeBackend(**backend_kw(max_tokens=B, device=local_rank, cache_gb=args.cache_gb))
    be.synthesize(SEED, SIGMA, SIGMA)
    P = 64
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    pool = torch.randn((P, B, D_), generator=g, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    for i in range(max(args.warmup, 3)):
        be.forward_dev(pool[i % P], B, stream=stream)
        be.tick()
    be.sync(stream)
    be.reset_stats()
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for i in range(args.steps):
        be.forward_dev(pool[i % P], B, stream=stream)
        be.tick()
    e1.record(stream)
    be.sync(stream)
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    st = be.stats()
    value = args.steps * B / (ms / 1000.0)
    hbm, peak_kind = peaks()
    uses = max(1, st["hits"] + st["misses"])
    line = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4xq8-int32+f32", "data": "synthetic",
            "config": dict(workload_config(B, 1), cache_gb=args.cache_gb,
                           store=f"{st['n_slots']} HBM slots for {L_ * E_} experts, LFU, next-layer prefetch"),
            "store": {"hit_rate": round(st["hits"] / uses, 4), "copies_per_step": round(st["copies"] / args.steps, 2),
                      "bytes_copied_per_step": round(st["bytes_copied"] / args.steps),
                      "prefetch_issued": st["prefetch_issued"], "prefetch_used": st["prefetch_used"],
                      "stall_s": round(st["stall_s"], 3)},
            "roofline": {"bound": "host link", "achieved": round(st["bytes_copied"] / (ms * 1e-3) / 1e9, 1),
                         "unit": "GB/s", "kernel": "host -> HBM expert copies (pinned host tier)",
                         "peak": None, "frac": None, "traffic": None},
            "cpu_baseline": None,
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                    "timing": "CUDA events; the store's host reads of the routing happen inside every step"},
            "gpu_launches": None, "clocks": clk}
    print(json.dumps(line), flush=True)
    be.close()


def run_ours(args, rank, world, local_rank):
    import torch
    import hearth_b200 as hb
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B = args.batch
    be = hb.MoeBackend(**backend_kw(max_tokens=B, device=local_rank))
    be.synthesize(SEED, SIGMA, SIGMA)
    # token pool resident in HBM; each step evaluates a fresh slot in place
    P = 64
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    pool = torch.randn((P, B, D_), generator=g, device=dev, dtype=torch.float32)
    # kernels and events on one stream: the torch stream object (its default stream is passed to the
    # library as the legacy default stream, not as "the library's own stream")
    stream = torch.cuda.current_stream(dev)
    sp = stream
    for i in range(max(args.warmup, 3)):
        be.forward_dev(pool[i % P], B, stream=sp)
    for i in range(P):                                   # every pool slot's graph exists before timing
        be.forward_dev(pool[i], B, stream=sp)
    be.sync(sp)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for i in range(args.steps):
        be.forward_dev(pool[i % P], B, stream=sp)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    be.sync(sp)
    ms = e0.elapsed_time(e1)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ms, world, dev)
    value = world * args.steps * B / (ms / 1000.0)
    assert torch.isfinite(pool).all().item()

    # ---- end to end through the public C ABI with host buffers
    rng = np.random.default_rng(7 + rank)
    host = [np.ascontiguousarray(rng.standard_normal((B, D_)).astype(np.float32)) for _ in range(P)]
    for i in range(3):
        be.forward_into(host[i])
    e2e_steps = min(args.steps, 2000)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        be.forward_into(host[i % P])
    t_e2e = time.perf_counter() - t0
    t_e2e = max_over_ranks(t_e2e, world, dev)
    e2e = world * e2e_steps * B / t_e2e

    # ---- roofline of the dominant kernel, timed live with CUDA events on its launching stream.
    # Batch 1 runs a persistent decode kernel: one launch per step covers every layer, so
    # its average launch duration is the timed region / steps. Other batches run the per-stage
    # kernels; their dominant one is k_moe_gateup, timed by hxb_moe_profile.
    us = be.profile(B, 2)
    ab = algorithmic_bytes()
    hbm, peak_kind = peaks()
    step_gbs = step_bytes(B) / (ms / args.steps * 1e-3) / 1e9
    path = be.decode_path()
    persistent = B == 1 and path != "layers"
    if persistent:
        kernel = "k_moe_decode (persistent, one launch per token, all layers)"
        kbytes, kgbs = L_ * ab["layer"], step_gbs
    elif B * K_ >= 256:
        kernel = ("k_moe_gateup_ws (staged tcgen05 gate+up over expert buckets, SwiGLU, mid act-quant; "
                  "time from hxb_moe_profile)")
        kbytes = batch_gateup_bytes(B)
        kgbs = kbytes / (us[2] * 1e-6) / 1e9
    else:
        kernel, kbytes = "k_moe_gateup (Q4 gate+up GEMV, SwiGLU, mid act-quant)", ab["gateup"]
        kgbs = ab["gateup"] / (us[2] * 1e-6) / 1e9

    # ---- CPU baseline (rank 0, N = 1): reference kernels on the host, same weights; and a full-size
    # bit-exact spot check of the GPU against it on the sampled tokens
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu and MODEL != "kimi":
        from oracle import oracle as O
        if O.moe_ref_lib() is not None:
            ref = O.MoeRef(n_threads=0)
            model, _ = cpu_model(ref, L_)
            arr = model.c_layers()
            tps, n, ins, outs = time_cpu(ref, model, arr, B, 20.0, 400, np.random.default_rng(99))
            cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": ref.threads, "kind": "reference",
                   "sample": f"{n} decode steps of batch {B} (~20 s) of the same {L_}-layer workload, reference "
                             f"AVX-512 kernels + hx_pool on {ref.threads} threads"}
            bad = 0
            for hin, hout in zip(ins[:16], outs[:16]):
                g_ = be.forward(hin)
                bad += int(not np.array_equal(g_.view(np.uint32), hout.view(np.uint32)))
            parity = f"{min(16, len(ins)) - bad}/{min(16, len(ins))} decode steps bit-identical to the CPU reference"
            ref.close()
        else:
            cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
                   "sample": "oracle/_ref not built"}

    # per layer: norm+act, router (fused routing), gate/up, down for B * K <= 64; otherwise norm+act,
    # router, select, union, gate/up, down, rank-order sum
    launches_per_step = 1 if persistent else (L_ * 4 if B * K_ <= 64 else L_ * 7)
    line = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4xq8-int32+f32", "data": "synthetic",
            "config": workload_config(B, world),
            "roofline": {"bound": "hbm", "achieved": round(kgbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(kgbs / hbm, 4),
                         "traffic": round(DECODE_DRAM_BYTES_PER_LAYER * L_) if persistent and MODEL == "qwen3"
                         else None,
                         "traffic_note": ("ncu dram bytes of a 4-layer capture scaled to the launch's layers"
                                          if persistent else None),
                         "kernel": kernel, "peak_kind": peak_kind,
                         "multi_kernel_stage_us": {"norm_act": round(us[0], 3), "router": round(us[1], 3),
                                                   "gateup": round(us[2], 3), "down": round(us[3], 3)},
                         "bytes_per_launch": kbytes,
                         "step_bytes": step_bytes(B), "step_gbs": round(step_gbs, 1),
                         "step_frac": round(step_gbs / hbm, 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": B * D_ * 4,
                    "d2h_bytes_per_step": B * D_ * 4 + 4, "timing": "host clock around synchronous hxb_moe_forward"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk}
    if parity:
        line["parity"] = parity
    if rank == 0:
        print(json.dumps(line), flush=True)
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3", choices=sorted(MODELS),
                    help="the MoE stack: qwen3 (Qwen3-30B-A3B, the headline), olmoe (OLMoE-1B-7B), mixtral "
                         "(Mixtral-8x7B, batch 8 by default), kimi (Kimi-K2: sigmoid grouped router with bias, "
                         "Q8 shared expert; expert-parallel over >= 4 GPUs for all 60 MoE layers)")
    ap.add_argument("--batch", type=int, default=None, help="tokens per step (default: the model's configuration)")
    ap.add_argument("--layers", type=int, default=None, help="MoE layers (default: the model's, or as many as fit "
                                                              "the GPUs' HBM); fewer for small profiling captures")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: N independent replicas of the stack, one per GPU (weak scaling) instead of the "
                         "default expert parallelism (one token stream, expert e on rank e %% N: strong scaling)")
    ap.add_argument("--cache-gb", type=float, default=0.0,
                    help="HBM budget for expert slots below the stack's experts: the streaming store path")
    ap.add_argument("--full", action="store_true",
                    help="the whole decoder (embedding, GQA attention + KV cache, MoE, LM head) of qwen3 / olmoe / "
                         "mixtral on one GPU, decode steps after a 512-token prompt")
    ap.add_argument("--trace", action="store_true",
                    help="instead of the bench line: the persistent kernel's per-phase timeline (mean us per "
                         "layer over CTAs, thread 0's SM clock) as one JSON line")
    args = ap.parse_args()
    rank, world, local_rank = dist_env()
    set_model(args.model, args.layers, 1 if args.replicas else world)
    if args.batch is None:
        args.batch = MODELS[args.model]["batch"]
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        # the line is the only thing on stdout: native code (the communicator set-up prints its NCCL
        # version there) writes to stderr from here on, Python's stdout keeps the original descriptor
        sys.stdout.flush()
        real_out = os.dup(1)
        os.dup2(2, 1)
        sys.stdout = os.fdopen(real_out, "w", buffering=1)
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.trace:
            if rank == 0:
                run_trace(args, local_rank)
        elif args.full:
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable": "the reference engine needs a container of "
                                                                          "the whole model, not written on the GPU box"}))
            elif rank == 0:
                run_full(args, rank, world, local_rank)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        elif args.cache_gb > 0:
            if rank == 0:
                run_stream(args, rank, world, local_rank)
        elif world > 1 and not args.replicas:
            run_ep(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
