"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checker and the CPU baseline.

* ``lib()``      -> oracle/liboracle.so, the C restatement of the reference's quantized MoE path
                    (hx_oracle.c; pinned to the reference's FNV-1a hashes, see tests/).
* ``ref_lib()``  -> oracle/_ref/libhearth_ref.so, the reference engine compiled from its own
                    sources (hearth_quantize / hearth_matmul / hearth_dequantize), or None.
* ``moe_ref_lib()`` -> oracle/_ref/libmoe_ref.so, the reference's AVX-512 kernels + thread pool
                    driven by moe_ref.c (the timed CPU baseline), or None.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32, F16, BF16, Q8, Q4 = 0, 1, 2, 3, 4
SOFTMAX, SIGMOID = 0, 1

_lib = None
_ref = None
_moe_ref = None


def reference_tree():
    """The reference checkout to compile _ref/ from: $HEARTH_REF, else a checkout named `reference`
    beside this repository; None when neither holds the engine sources (e.g. on a GPU box, which only
    uses the prebuilt _ref/)."""
    for cand in (os.environ.get("HEARTH_REF"), os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "engine", "src")):
            return cand
    return None


def build(quiet: bool = True) -> None:
    """Build liboracle.so and, where the reference tree exists, _ref/ (make -C oracle REF=...)."""
    cmd = ["make", "-C", HERE, "-j8"]
    ref = reference_tree()
    if ref:
        cmd.append(f"REF={ref}")
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


class RouteCfg(C.Structure):
    _fields_ = [("E", C.c_int), ("K", C.c_int), ("score_fn", C.c_int), ("score_bias", C.c_int),
                ("n_group", C.c_int), ("topk_group", C.c_int), ("norm_topk_prob", C.c_int),
                ("routed_scale", C.c_float)]


class MoeLayer(C.Structure):
    _fields_ = [("D", C.c_int), ("F", C.c_int), ("route", RouteCfg),
                ("router", C.c_void_p), ("router_bias", C.c_void_p),
                ("slabs", C.c_void_p), ("slab_dtype", C.c_void_p),
                ("Fs", C.c_int), ("sh_dtype", C.c_int),
                ("sh_gate", C.c_void_p), ("sh_up", C.c_void_p), ("sh_down", C.c_void_p),
                ("sh_gate_inp", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("eps", C.c_float), ("residual_scale", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_row_bytes.restype = C.c_size_t
        L.orc_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.orc_f16.restype = C.c_float
        L.orc_f16.argtypes = [C.c_uint16]
        L.orc_fnv1a.restype = C.c_uint64
        L.orc_fnv1a.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]
        L.orc_det_fill.argtypes = [C.c_void_p, C.c_int64, C.c_uint64]
        L.orc_expf_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.orc_act_quantize.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.orc_matmul.restype = C.c_int
        L.orc_matmul.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int, C.c_void_p]
        L.orc_dequantize.restype = C.c_int
        L.orc_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
        L.orc_route_select.argtypes = [C.POINTER(RouteCfg), C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_route_weights.argtypes = [C.POINTER(RouteCfg), C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_route_union.restype = C.c_int
        L.orc_route_union.argtypes = [C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 6
        L.orc_slab_layout.argtypes = [C.c_int, C.c_int64, C.c_int64, C.POINTER(C.c_size_t),
                                      C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        L.orc_moe_layer_eval.restype = C.c_int
        L.orc_moe_layer_eval.argtypes = [C.POINTER(MoeLayer), C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_moe_forward.restype = C.c_int
        L.orc_moe_forward.argtypes = [C.POINTER(MoeLayer), C.c_int, C.c_void_p, C.c_int]
        _lib = L
    return _lib


def ref_lib():
    """The reference engine built from its sources, or None where it was never built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libhearth_ref.so")
        if not os.path.exists(path):
            if reference_tree():
                build()
            if not os.path.exists(path):
                return None
        L = C.CDLL(path)
        L.hearth_quantize.restype = C.c_int
        L.hearth_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int]
        L.hearth_matmul.restype = C.c_int
        L.hearth_matmul.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        L.hearth_dequantize.restype = C.c_int
        L.hearth_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
        L.hearth_row_bytes.restype = C.c_size_t
        L.hearth_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.hearth_cpu_isa.restype = C.c_int
        _ref = L
    return _ref


def moe_ref_lib():
    global _moe_ref
    if _moe_ref is None:
        path = os.path.join(HERE, "_ref", "libmoe_ref.so")
        if not os.path.exists(path):
            if reference_tree():
                build()
            if not os.path.exists(path):
                return None
        L = C.CDLL(path)
        L.moe_ref_open.restype = C.c_void_p
        L.moe_ref_open.argtypes = [C.c_int, C.c_int]
        L.moe_ref_close.argtypes = [C.c_void_p]
        L.moe_ref_threads.restype = C.c_int
        L.moe_ref_threads.argtypes = [C.c_void_p]
        L.moe_ref_isa.restype = C.c_int
        L.moe_ref_isa.argtypes = [C.c_void_p]
        L.moe_ref_layer.restype = C.c_int
        L.moe_ref_layer.argtypes = [C.c_void_p, C.POINTER(MoeLayer), C.c_void_p, C.c_int, C.c_void_p]
        L.moe_ref_forward.restype = C.c_int
        L.moe_ref_forward.argtypes = [C.c_void_p, C.POINTER(MoeLayer), C.c_int, C.c_void_p, C.c_int]
        L.moe_ref_synth_q4.restype = C.c_int
        L.moe_ref_synth_q4.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_uint64,
                                       C.c_float]
        L.moe_ref_synth_f32.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_float]
        L.moe_ref_synth_blocks.restype = C.c_int
        L.moe_ref_synth_blocks.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_uint64, C.c_float]
        _moe_ref = L
    return _moe_ref


# ---------------------------------------------------------------- numpy conveniences

def row_bytes(dtype: int, n: int) -> int:
    return int(lib().orc_row_bytes(dtype, n))


def fnv1a(a: np.ndarray, h: int = 0xcbf29ce484222325) -> int:
    a = np.ascontiguousarray(a)
    return int(lib().orc_fnv1a(_p(a), a.nbytes, h))


def det_fill(n: int, seed: int) -> np.ndarray:
    x = np.empty(n, np.float32)
    lib().orc_det_fill(_p(x), n, seed)
    return x


def host_expf(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_expf_batch(_p(x), _p(y), x.size)
    return y


def act_quantize(x: np.ndarray) -> np.ndarray:
    """NUMERICS §2 activation blocks of x [.., n] as raw bytes [.., n/64*72]."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    rows = x.size // n
    out = np.zeros((rows, n // 64 * 72), np.uint8)
    for r in range(rows):
        lib().orc_act_quantize(_p(x.reshape(rows, n)[r]), _p(out[r]), n)
    return out.reshape(x.shape[:-1] + (n // 64 * 72,))


def matmul(dtype: int, W: np.ndarray, n_rows: int, n_cols: int, X: np.ndarray) -> np.ndarray:
    X = np.ascontiguousarray(X, np.float32).reshape(-1, n_cols)
    W = np.ascontiguousarray(W)
    Y = np.empty((X.shape[0], n_rows), np.float32)
    rc = lib().orc_matmul(dtype, _p(W), n_rows, n_cols, _p(X), X.shape[0], _p(Y))
    if rc:
        raise ValueError(f"orc_matmul returned {rc}")
    return Y


def dequantize(dtype: int, W: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    out = np.empty((n_rows, n_cols), np.float32)
    rc = lib().orc_dequantize(dtype, _p(np.ascontiguousarray(W)), n_rows, n_cols, _p(out))
    if rc:
        raise ValueError(f"orc_dequantize returned {rc}")
    return out


def ref_quantize(dtype: int, W: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """The reference's own quantizer (hearth_quantize) on W [rows, cols] f32."""
    L = ref_lib()
    if L is None:
        raise RuntimeError("reference library not built (oracle/_ref/libhearth_ref.so)")
    W = np.ascontiguousarray(W, np.float32)
    rows, cols = W.shape
    out = np.empty(rows * int(L.hearth_row_bytes(dtype, cols)), np.uint8)
    if L.hearth_quantize(dtype, _p(W), rows, cols, _p(out), n_threads) != 0:
        raise ValueError("hearth_quantize failed")
    return out.reshape(rows, -1)


def slab_layout(dtype: int, D: int, F: int):
    up, down, nb = C.c_size_t(), C.c_size_t(), C.c_size_t()
    lib().orc_slab_layout(dtype, D, F, C.byref(up), C.byref(down), C.byref(nb))
    return up.value, down.value, nb.value


class MoeModel:
    """Numpy-held weights of one or more MoE layers, laid out as the CUDA backend expects."""

    def __init__(self, D, F, E, K, *, score_fn=SOFTMAX, score_bias=0, n_group=1, topk_group=1,
                 norm_topk_prob=1, routed_scale=1.0, eps=1e-6, residual_scale=1.0):
        self.D, self.F, self.E, self.K = D, F, E, K
        self.route = dict(score_fn=score_fn, score_bias=score_bias, n_group=n_group, topk_group=topk_group,
                          norm_topk_prob=norm_topk_prob, routed_scale=routed_scale)
        self.eps, self.residual_scale = eps, residual_scale
        self.layers = []   # dicts: router, bias, slabs [E] uint8 arrays, dtypes [E], ffn_norm, shared
        self._keep = []

    def add_layer(self, router, slabs, dtypes, ffn_norm=None, bias=None, shared=None):
        self.layers.append(dict(router=np.ascontiguousarray(router, np.float32),
                                bias=None if bias is None else np.ascontiguousarray(bias, np.float32),
                                slabs=[np.ascontiguousarray(s) for s in slabs],
                                dtypes=np.ascontiguousarray(dtypes, np.int32),
                                ffn_norm=np.ones(self.D, np.float32) if ffn_norm is None
                                else np.ascontiguousarray(ffn_norm, np.float32),
                                shared=shared))

    def c_layers(self):
        arr = (MoeLayer * len(self.layers))()
        keep = []
        for i, l in enumerate(self.layers):
            ptrs = (C.c_void_p * self.E)(*[s.ctypes.data for s in l["slabs"]])
            keep.append(ptrs)
            c = arr[i]
            c.D, c.F = self.D, self.F
            c.route = RouteCfg(self.E, self.K, self.route["score_fn"], self.route["score_bias"],
                               self.route["n_group"], self.route["topk_group"], self.route["norm_topk_prob"],
                               self.route["routed_scale"])
            c.router = l["router"].ctypes.data
            c.router_bias = l["bias"].ctypes.data if l["bias"] is not None else None
            c.slabs = C.cast(ptrs, C.c_void_p).value
            c.slab_dtype = l["dtypes"].ctypes.data
            sh = l["shared"]
            if sh is not None:
                c.Fs, c.sh_dtype = sh["Fs"], sh["dtype"]
                c.sh_gate, c.sh_up, c.sh_down = sh["gate"].ctypes.data, sh["up"].ctypes.data, sh["down"].ctypes.data
                c.sh_gate_inp = sh["gate_inp"].ctypes.data if sh.get("gate_inp") is not None else None
            else:
                c.Fs, c.sh_dtype = 0, 0
            c.ffn_norm = l["ffn_norm"].ctypes.data
            c.eps, c.residual_scale = self.eps, self.residual_scale
        self._keep = keep
        return arr

    def layer_eval(self, layer: int, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        arr = self.c_layers()
        out = np.empty((T, self.D), np.float32)
        ids = np.empty((T, self.K), np.int32)
        w = np.empty((T, self.K), np.float32)
        rc = lib().orc_moe_layer_eval(C.byref(arr[layer]), _p(x), T, _p(out), _p(ids), _p(w))
        if rc:
            raise ValueError(f"orc_moe_layer_eval returned {rc}")
        return out, ids, w

    def forward(self, h: np.ndarray, layer0: int = 0, n_layers: int | None = None):
        h = np.array(h, np.float32, copy=True, order="C")
        arr = self.c_layers()
        n = len(self.layers) - layer0 if n_layers is None else n_layers
        rc = lib().orc_moe_forward(C.byref(arr[layer0]), n, _p(h), h.shape[0])
        if rc:
            raise ValueError(f"orc_moe_forward returned {rc}")
        return h


class MoeRef:
    """The timed CPU baseline: the reference's kernels and pool over all host cores."""

    def __init__(self, n_threads: int = 0, isa: int = 0):
        L = moe_ref_lib()
        if L is None:
            raise RuntimeError("oracle/_ref/libmoe_ref.so not built")
        self.L = L
        self.h = L.moe_ref_open(n_threads, isa)
        if not self.h:
            raise RuntimeError("moe_ref_open failed")

    @property
    def threads(self) -> int:
        return int(self.L.moe_ref_threads(self.h))

    @property
    def isa(self) -> int:
        return int(self.L.moe_ref_isa(self.h))

    def layer(self, model: MoeModel, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        arr = model.c_layers()
        out = np.empty_like(x)
        rc = self.L.moe_ref_layer(self.h, C.byref(arr[layer]), _p(x), x.shape[0], _p(out))
        if rc:
            raise ValueError(f"moe_ref_layer returned {rc}")
        return out

    def forward(self, model: MoeModel, h: np.ndarray, arr=None) -> np.ndarray:
        if arr is None:
            arr = model.c_layers()
        rc = self.L.moe_ref_forward(self.h, arr, len(model.layers), _p(h), h.shape[0])
        if rc:
            raise ValueError(f"moe_ref_forward returned {rc}")
        return h

    def synth_q4(self, n_slabs: int, slab_bytes: int, D: int, F: int, seed: int, sigma: float) -> np.ndarray:
        """Expert slabs byte-identical to the backend's device generator (hxb_moe_synthesize)."""
        out = np.empty((n_slabs, slab_bytes), np.uint8)
        if self.L.moe_ref_synth_q4(self.h, out.ctypes.data, n_slabs, slab_bytes, D, F, seed, sigma):
            raise ValueError("moe_ref_synth_q4 failed")
        return out

    def synth_f32(self, n: int, seed: int, sigma: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.moe_ref_synth_f32(out.ctypes.data, n, seed, sigma)
        return out

    def synth_blocks(self, dtype: int, rows: int, cols: int, seed: int, sigma: float) -> np.ndarray:
        """A [rows, row_bytes] Q4/Q8 matrix byte-identical to the backend's device generator of shared
        experts (hxb_moe_synthesize)."""
        out = np.empty((rows, row_bytes(dtype, cols)), np.uint8)
        if self.L.moe_ref_synth_blocks(out.ctypes.data, dtype, rows, cols, seed, sigma):
            raise ValueError("moe_ref_synth_blocks failed")
        return out

    def close(self):
        if self.h:
            self.L.moe_ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
