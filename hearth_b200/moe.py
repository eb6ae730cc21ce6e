"""Host-side handle of the MoE backend: the quantized expert path of the reference's
``moe_layer`` (engine/src/model.c:986-1131) with its expert store, on one GPU.

Weights come from numpy buffers laid out like the .hearth container (docs/FORMAT.md §5 slabs,
row-major [out, in] matrices), or are synthesised in HBM for benchmarks.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import COPY_HOOK, MoeConfig, MoeStats, check, lib


def _ptr(a):
    if a is None:
        return None
    if hasattr(a, "data_ptr"):          # a torch tensor (device buffers for the *_dev calls)
        return C.c_void_p(a.data_ptr())
    return C.c_void_p(a.ctypes.data)


_CUDA_STREAM_LEGACY = 1   # cudaStreamLegacy: the legacy default stream, as a stream handle


def _stream(s):
    """Stream argument of the *_dev calls. None or 0: the library's own stream. A torch.cuda.Stream:
    that stream (torch's default stream maps to the legacy default stream, so the work orders with
    what torch issues there). Anything else: a raw cudaStream_t handle."""
    if s is None:
        return C.c_void_p(0)
    if hasattr(s, "cuda_stream"):
        return C.c_void_p(s.cuda_stream or _CUDA_STREAM_LEGACY)
    return C.c_void_p(int(s))


_CONFIG_KEYS = ("n_layers", "d_model", "expert_ffn_dim", "n_experts", "top_k", "score_fn", "score_bias", "n_group",
                "topk_group", "norm_topk_prob", "routed_scale", "residual_scale", "norm_eps", "expert_dtype",
                "shared_ffn_dim", "shared_dtype", "shared_gate")


def container_probe(path) -> tuple[dict, dict]:
    """Reads and validates a .hearth container (host only): (the MoeBackend configuration of its MoE
    path, {n_layers, n_moe_layers, n_expert_entries, n_physical_slabs, n_aliased, expert_dtype,
    slab_bytes}). Raises ValueError for a file that breaks the format, OSError for one that cannot be
    read."""
    from ._lib import ContainerInfo
    c, info = MoeConfig(), ContainerInfo()
    err = C.create_string_buffer(512)
    rc = lib().hxb_container_probe(os.fsencode(path), C.byref(c), C.byref(info), err, 512)
    if rc == _lib.HXB_E_IO:
        raise OSError(err.value.decode())
    if rc != 0:
        raise ValueError(err.value.decode())
    cfg = {k: getattr(c, k) for k in _CONFIG_KEYS}
    return cfg, {k: getattr(info, k) for k, _ in info._fields_}


class MoeBackend:
    """One MoE stack (n_layers layers of the same shape) on one CUDA device."""

    @classmethod
    def from_container(cls, path, **options) -> "MoeBackend":
        """A handle for a .hearth container's MoE layers (one slot per model layer; dense layers stay
        unset) with its weights loaded. options: max_tokens, cache_gb, policy, heat_decay, device,
        ep_size, ep_rank."""
        cfg, _ = container_probe(path)
        b = cls(**cfg, **options)
        try:
            b.load_container(path)
        except BaseException:
            b.close()
            raise
        return b

    def load_container(self, path) -> None:
        check(lib().hxb_moe_load_container(self.h, os.fsencode(path)), "hxb_moe_load_container")

    def __init__(self, *, n_layers: int, d_model: int, expert_ffn_dim: int, n_experts: int, top_k: int,
                 score_fn: int = 0, score_bias: int = 0, n_group: int = 1, topk_group: int = 1,
                 norm_topk_prob: int = 1, routed_scale: float = 1.0, residual_scale: float = 1.0,
                 norm_eps: float = 1e-6, expert_dtype: int = _lib.Q4, shared_ffn_dim: int = 0,
                 shared_dtype: int = _lib.Q8, shared_gate: int = 0, max_tokens: int = 1, cache_gb: float = 0.0,
                 policy: int = _lib.POLICY_LFU, heat_decay: float = 0.995, device: int = 0, ep_size: int = 1,
                 ep_rank: int = 0, prefetch_next: int = 1):
        L = lib()
        c = MoeConfig()
        L.hxb_moe_default_config(C.byref(c))
        for k, v in dict(n_layers=n_layers, d_model=d_model, expert_ffn_dim=expert_ffn_dim, n_experts=n_experts,
                         top_k=top_k, score_fn=score_fn, score_bias=score_bias, n_group=n_group,
                         topk_group=topk_group, norm_topk_prob=norm_topk_prob, routed_scale=routed_scale,
                         residual_scale=residual_scale, norm_eps=norm_eps, expert_dtype=expert_dtype,
                         shared_ffn_dim=shared_ffn_dim, shared_dtype=shared_dtype, shared_gate=shared_gate,
                         max_tokens=max_tokens, cache_gb=cache_gb, policy=policy, heat_decay=heat_decay,
                         device=device, ep_size=ep_size, ep_rank=ep_rank, prefetch_next=prefetch_next).items():
            setattr(c, k, v)
        err = C.create_string_buffer(512)
        h = L.hxb_moe_open(C.byref(c), err, 512)
        if not h:
            raise RuntimeError(f"hxb_moe_open failed: {err.value.decode()}")
        self.h = h
        self.cfg = c
        self.D, self.F, self.E, self.K = d_model, expert_ffn_dim, n_experts, top_k
        self.n_layers = n_layers
        self.ep_size, self.ep_rank = ep_size, ep_rank
        self._hook = None

    # ------------------------------------------------------------------ weights
    @property
    def slab_bytes(self) -> int:
        return int(lib().hxb_moe_slab_bytes(self.h))

    def set_layer(self, layer: int, router: np.ndarray, router_bias=None, ffn_norm=None, sh_gate=None, sh_up=None,
                  sh_down=None, sh_gate_inp=None) -> None:
        router = np.ascontiguousarray(router, np.float32)
        assert router.shape == (self.E, self.D)
        keep = [router]
        args = []
        for a, dt in ((router_bias, np.float32), (ffn_norm, np.float32), (sh_gate, None), (sh_up, None),
                      (sh_down, None), (sh_gate_inp, np.float32)):
            if a is None:
                args.append(None)
            else:
                a = np.ascontiguousarray(a, dt) if dt is not None else np.ascontiguousarray(a)
                keep.append(a)
                args.append(_ptr(a))
        check(lib().hxb_moe_set_layer(self.h, layer, _ptr(router), *args), "hxb_moe_set_layer")

    def set_expert(self, layer: int, expert: int, slab: np.ndarray) -> None:
        slab = np.ascontiguousarray(slab, np.uint8)
        check(lib().hxb_moe_set_expert(self.h, layer, expert, _ptr(slab), slab.nbytes), "hxb_moe_set_expert")

    def share_expert(self, layer: int, expert: int, src_layer: int, src_expert: int) -> None:
        """(layer, expert) uses the pinned host copy of (src_layer, src_expert)'s slab (an aliased
        container entry); it keeps its own HBM slot and counters."""
        check(lib().hxb_moe_share_expert(self.h, layer, expert, src_layer, src_expert), "hxb_moe_share_expert")

    def synthesize(self, seed: int = 0, sigma_router: float = 0.02, sigma_expert: float = 0.02) -> None:
        check(lib().hxb_moe_synthesize(self.h, seed, sigma_router, sigma_expert), "hxb_moe_synthesize")

    # ------------------------------------------------------------------ evaluation
    def forward(self, h: np.ndarray, layer0: int = 0, n_layers: int | None = None) -> np.ndarray:
        """h [T, D] (host): for each layer, h = h + rs * moe(rmsnorm(h)). Returns a new array."""
        n_layers = self.n_layers - layer0 if n_layers is None else n_layers
        out = np.array(h, dtype=np.float32, copy=True, order="C")
        check(lib().hxb_moe_forward(self.h, _ptr(out), out.shape[0], layer0, n_layers), "hxb_moe_forward")
        return out

    def forward_routed(self, h: np.ndarray, ids: np.ndarray, layer0: int = 0) -> np.ndarray:
        """Route replay: like forward, with every token's K expert ids of every layer given
        (ids [n_layers, T, K]); scores and weights computed as usual. Returns a new array."""
        out = np.array(h, dtype=np.float32, copy=True, order="C")
        ids = np.ascontiguousarray(ids, np.int32)
        assert ids.ndim == 3 and ids.shape[1:] == (out.shape[0], self.K)
        check(lib().hxb_moe_forward_routed(self.h, _ptr(out), out.shape[0], layer0, ids.shape[0], _ptr(ids)),
              "hxb_moe_forward_routed")
        return out

    def forward_into(self, h: np.ndarray, layer0: int = 0, n_layers: int | None = None) -> None:
        """In place on a C-contiguous float32 host array (no copies beyond the library's)."""
        n_layers = self.n_layers - layer0 if n_layers is None else n_layers
        check(lib().hxb_moe_forward(self.h, _ptr(h), h.shape[0], layer0, n_layers), "hxb_moe_forward")

    def forward_dev(self, h, T: int, layer0: int = 0, n_layers: int | None = None, stream=None) -> None:
        """h: device buffer (torch tensor or raw pointer) of [T, D] float32, updated in place."""
        n_layers = self.n_layers - layer0 if n_layers is None else n_layers
        hp = _ptr(h) if hasattr(h, "data_ptr") else C.c_void_p(int(h))
        check(lib().hxb_moe_forward_dev(self.h, hp, T, layer0, n_layers, _stream(stream)),
              "hxb_moe_forward_dev")

    def sync(self, stream=None) -> None:
        """Waits for the stream of the *_dev calls and raises on a device-side error."""
        check(lib().hxb_moe_sync(self.h, _stream(stream)), "hxb_moe_sync")

    # ------------------------------------------------------------------ expert parallelism
    def owns(self, expert: int) -> bool:
        """This handle holds and computes `expert` (expert e lives on rank e % ep_size)."""
        return expert % self.ep_size == self.ep_rank

    def ep_layer_dev(self, layer: int, h, T: int, y, stream=None) -> None:
        """Expert parallelism, step 1: routing of the T tokens of h [T, D] and the outputs of this
        rank's (token, rank) pairs into y [T*K, D] (device buffers); see hxb_moe_ep_layer_dev."""
        check(lib().hxb_moe_ep_layer_dev(self.h, layer, _ptr(h), T, _ptr(y), _stream(stream)), "hxb_moe_ep_layer_dev")

    def ep_combine_dev(self, layer: int, y_all, T: int, h, stream=None) -> None:
        """Expert parallelism, step 2: h += rs * rank-order sum over y_all [ep_size, T*K, D]."""
        check(lib().hxb_moe_ep_combine_dev(self.h, layer, _ptr(y_all), T, _ptr(h), _stream(stream)),
              "hxb_moe_ep_combine_dev")

    def decode_path(self) -> str:
        """Kernel of a single-token forward over every layer: "layers" (per-phase kernels) or
        "persistent" (one launch for all layers)."""
        return ("layers", "persistent")[lib().hxb_moe_decode_path(self.h)]

    def phase_trace(self):
        """Phase timeline of the last single-token persistent launch (handle opened with the
        environment variable HXB_TRACE=1): uint64 array [layers, CTAs, stamps] of SM clock cycles,
        or None when not tracing."""
        n = lib().hxb_moe_phase_trace(self.h, None, 0)
        if n <= 0:
            return None
        buf = np.zeros(n, np.uint64)
        if lib().hxb_moe_phase_trace(self.h, C.c_void_p(buf.ctypes.data), n) != n:
            raise RuntimeError("hxb_moe_phase_trace failed")
        return buf

    def profile(self, T: int = 1, iters: int = 3) -> list:
        """Average device microseconds per stage of one layer: [norm+act, router, gate/up, down]."""
        us = (C.c_double * 4)()
        check(lib().hxb_moe_profile(self.h, T, iters, us), "hxb_moe_profile")
        return list(us)

    def layer(self, layer: int, x: np.ndarray) -> np.ndarray:
        """One MoE FFN on x [T, D] as given: the rank-order expert sum [T, D]."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        check(lib().hxb_moe_layer(self.h, layer, _ptr(x), x.shape[0], _ptr(out)), "hxb_moe_layer")
        return out

    def layer_dev(self, layer: int, x, out, T: int, stream=None) -> None:
        check(lib().hxb_moe_layer_dev(self.h, layer, _ptr(x), T, _ptr(out), _stream(stream)),
              "hxb_moe_layer_dev")

    def last_routing(self, T: int):
        ids = np.empty((T, self.K), np.int32)
        w = np.empty((T, self.K), np.float32)
        check(lib().hxb_moe_last_routing(self.h, _ptr(ids), _ptr(w), T), "hxb_moe_last_routing")
        return ids, w

    # ------------------------------------------------------------------ store
    def get_expert(self, layer: int, expert: int, out=None):
        """The expert's slab bytes as this (resident) handle holds them in HBM."""
        n = int(lib().hxb_moe_slab_bytes(self.h))
        if out is None:
            out = np.empty(n, np.uint8)
        check(lib().hxb_moe_get_expert(self.h, layer, expert, out.ctypes.data, out.nbytes), "hxb_moe_get_expert")
        return out

    def stats(self) -> dict:
        s = MoeStats()
        check(lib().hxb_moe_get_stats(self.h, C.byref(s)), "hxb_moe_get_stats")
        return {k: getattr(s, k) for k, _ in MoeStats._fields_}

    def reset_stats(self) -> None:
        lib().hxb_moe_reset_stats(self.h)

    def is_resident(self, layer: int, expert: int) -> bool:
        return bool(lib().hxb_moe_is_resident(self.h, layer, expert))

    def tick(self) -> None:
        lib().hxb_moe_tick(self.h)

    def prefetch(self, layer: int, experts) -> None:
        a = np.ascontiguousarray(experts, np.int32)
        check(lib().hxb_moe_prefetch(self.h, layer, _ptr(a), a.size), "hxb_moe_prefetch")

    def seed_heat(self, counts: np.ndarray, pin_fraction: float = 0.0, warm_start: bool = False) -> None:
        c = np.ascontiguousarray(counts, np.float32)
        check(lib().hxb_moe_seed_heat(self.h, _ptr(c), c.size, pin_fraction, int(warm_start)), "hxb_moe_seed_heat")

    def set_copy_hook(self, fn) -> None:
        """fn(layer, expert) -> int; nonzero fails that host->HBM copy (test seam)."""
        if fn is None:
            self._hook = None
            lib().hxb_moe_set_copy_hook(self.h, COPY_HOOK(), None)
            return
        self._hook = COPY_HOOK(lambda ctx, l, e: int(fn(l, e)))
        lib().hxb_moe_set_copy_hook(self.h, self._hook, None)

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hxb_moe_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
