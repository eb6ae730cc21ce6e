"""The whole decoder on the GPU (hxb_model_*): a container evaluated the way the reference engine's
public API evaluates it (engine/include/hearth.h hearth_eval, engine/src/model.c:1280-1332
hx_model_eval and 1171-1236 forward): tokens go through the embedding, every layer's attention with
its KV cache and its MoE or dense FFN, the output norm and the LM head on one B200, and the logits
equal the reference's bit for bit.

    with Model("model.hearth") as m:
        logits = m.eval(prompt, all_logits=True)     # [n, V]
        nxt = m.eval([int(logits[-1].argmax())])     # [V]
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import check, lib
from .moe import _stream


class _Synthetic:
    def __init__(self, arch, seed):
        self.arch, self.seed = arch, seed


class Model:
    def __init__(self, path: str, *, device: int = 0, max_batch: int = 0, max_seq: int = 0, cache_gb: float = 0.0,
                 policy: int = _lib.POLICY_LFU):
        L = lib()
        o = _lib.ModelOptions()
        L.hxb_model_default_options(C.byref(o))
        o.device, o.max_batch, o.max_seq, o.cache_gb, o.policy = device, max_batch, max_seq, cache_gb, policy
        err = C.create_string_buffer(512)
        if isinstance(path, _Synthetic):
            h = L.hxb_model_synthesize(C.byref(path.arch), C.byref(o), path.seed, err, 512)
        else:
            h = L.hxb_model_open(os.fsencode(path), C.byref(o), err, 512)
        if not h:
            raise RuntimeError(f"opening the model failed: {err.value.decode()}")
        self.h = h
        v = [C.c_int() for _ in range(6)]
        check(L.hxb_model_info(h, *[C.byref(x) for x in v]), "hxb_model_info")
        self.n_layers, self.d_model, self.vocab, self.max_seq, self.n_moe, self.top_k = (x.value for x in v)
        self.max_batch = max_batch or 512
        self.pos = 0
        self._routes = []

    @classmethod
    def synthesize(cls, *, vocab_size: int, n_heads: int, n_kv_heads: int, head_dim: int, qk_norm: int = 1,
                   rope_theta: float = 1e6, dense_dtype: int = _lib.Q8, sigma_dense: float = 0.02, seed: int = 0,
                   device: int = 0, max_batch: int = 0, max_seq: int = 0, **moe) -> "Model":
        """A decoder whose every layer is MoE, generated in HBM (hxb_model_synthesize): moe holds the
        MoE layers' hxb_moe_config fields (n_layers, d_model, expert_ffn_dim, n_experts, top_k, routing)."""
        L = lib()
        a = _lib.ModelArch()
        L.hxb_moe_default_config(C.byref(a.moe))
        for k, v in moe.items():
            setattr(a.moe, k, v)
        a.vocab_size, a.n_heads, a.n_kv_heads, a.head_dim = vocab_size, n_heads, n_kv_heads, head_dim
        a.qk_norm, a.rope_theta, a.dense_dtype, a.sigma_dense = qk_norm, rope_theta, dense_dtype, sigma_dense
        return cls(_Synthetic(a, seed), device=device, max_batch=max_batch, max_seq=max_seq)

    def forward(self, tokens, pos0: int, mode: int) -> np.ndarray | None:
        """forward(): T tokens at positions pos0.. ; mode 0 none, 1 last row [V], 2 every row [T, V]."""
        t = np.ascontiguousarray(tokens, np.int32)
        T = t.size
        out = np.empty((T if mode == 2 else 1) * self.vocab, np.float32) if mode else None
        check(lib().hxb_model_forward(self.h, t.ctypes.data, T, pos0, out.ctypes.data if mode else None, mode),
              "hxb_model_forward")
        if mode == 2:
            return out.reshape(T, self.vocab)
        return out

    def forward_dev(self, tokens, pos0: int, mode: int, logits=None, stream=None) -> None:
        """forward() on torch CUDA tensors (tokens int32 [T], logits float32 [1 or T, V]), asynchronous
        on `stream` (a torch stream, its default stream meaning the legacy default stream; None: the
        handle's own)."""
        check(lib().hxb_model_forward_dev(self.h, tokens.data_ptr(), tokens.numel(), pos0,
                                          logits.data_ptr() if logits is not None else None, mode, _stream(stream)),
              "hxb_model_forward_dev")

    def sync(self, stream=None) -> None:
        check(lib().hxb_model_sync(self.h, _stream(stream)), "hxb_model_sync")

    def eval(self, tokens, all_logits: bool = False) -> np.ndarray:
        """hearth_eval: the tokens in chunks of max_batch from the current position; the last token's
        logits [V], or every token's [n, V]. On failure the position is left as it was."""
        t = np.ascontiguousarray(tokens, np.int32).reshape(-1)
        n = t.size
        if n == 0:
            raise ValueError("no tokens")
        start = self.pos
        rows, routes = [], []
        try:
            for off in range(0, n, self.max_batch):
                T = min(self.max_batch, n - off)
                mode = 2 if all_logits else (1 if off + T == n else 0)
                lg = self.forward(t[off:off + T], self.pos, mode)
                if self.n_moe:
                    routes.append(self.last_routes(T))
                if mode == 2:
                    rows.append(lg)
                elif mode == 1:
                    rows = [lg]
                self.pos += T
        except Exception:
            self.pos = start
            raise
        self._routes = routes
        return np.concatenate(rows) if all_logits else rows[0]

    def last_routes(self, T: int) -> np.ndarray:
        """The last forward's routing rows [T, n_moe * K] (uint16, the FORMAT §9 trace rows)."""
        r = np.empty((T, self.n_moe * self.top_k), np.uint16)
        check(lib().hxb_model_last_routes(self.h, r.ctypes.data, T), "hxb_model_last_routes")
        return r

    def eval_routes(self) -> np.ndarray:
        """The routing rows of the last eval() (all its chunks)."""
        return np.concatenate(self._routes) if self._routes else np.empty((0, self.n_moe * self.top_k), np.uint16)

    def set_replay(self, rows) -> None:
        """Route replay from trace rows [n_rows, n_moe * K]; None stops it."""
        if rows is None:
            check(lib().hxb_model_set_replay(self.h, None, 0), "hxb_model_set_replay")
            return
        r = np.ascontiguousarray(rows, np.uint16)
        self._replay = r
        check(lib().hxb_model_set_replay(self.h, r.ctypes.data, r.shape[0]), "hxb_model_set_replay")

    def moe_stats(self) -> dict:
        """The MoE layers' counters (hxb_moe_get_stats of the handle inside)."""
        s = _lib.MoeStats()
        check(lib().hxb_moe_get_stats(lib().hxb_model_moe(self.h), C.byref(s)), "hxb_moe_get_stats")
        return {k: getattr(s, k) for k, _ in _lib.MoeStats._fields_}

    def reset(self) -> None:
        self.pos = 0

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hxb_model_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
