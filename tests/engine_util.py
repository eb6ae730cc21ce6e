"""ctypes access to the reference engine's public C API (engine/include/hearth.h:64-147: hearth_options,
hearth_open / hearth_eval / hearth_close, the routing trace), for the tests of the backend binding.
The struct mirrors the header field for field (the reference's own tests pin its layout,
python/tests/test_runtime.py). Two builds of the reference engine are used, both compiled from its
sources by oracle/Makefile: oracle/_ref/libhearth_ref.so (unchanged) and oracle/_ref/libhearth_cuda.so
(with the B200 binding oracle/hearth_cuda_backend.c: HEARTH_BACKEND=cuda puts the MoE layers on the
GPU)."""
import ctypes as C
import os

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(REPO, "oracle", "_ref", "libhearth_ref.so")
CUDA_LIB = os.path.join(REPO, "oracle", "_ref", "libhearth_cuda.so")
FIXTURE = os.path.join(REPO, "tests", "golden", "tiny_moe.hearth")


class HearthOptions(C.Structure):
    _fields_ = [("model_path", C.c_char_p), ("mirror_paths", C.c_char_p * 8), ("n_mirrors", C.c_int),
                ("cache_gb", C.c_double), ("n_threads", C.c_int), ("n_io_threads", C.c_int),
                ("direct_io", C.c_int), ("policy", C.c_int), ("prefetch", C.c_int), ("prefetch_extra", C.c_int),
                ("usage_in", C.c_char_p), ("usage_out", C.c_char_p), ("pin_fraction", C.c_float),
                ("warm_start", C.c_int), ("max_seq", C.c_int), ("max_batch", C.c_int), ("isa", C.c_int),
                ("verbose", C.c_int)]


class HearthModelInfo(C.Structure):
    _fields_ = [("arch", C.c_char * 32), ("n_layers", C.c_int), ("d_model", C.c_int), ("vocab_size", C.c_int),
                ("max_seq", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("attn_kind", C.c_int), ("n_experts", C.c_int), ("top_k", C.c_int), ("expert_ffn_dim", C.c_int),
                ("n_moe_layers", C.c_int), ("bos_id", C.c_int), ("n_eos", C.c_int), ("eos_ids", C.c_int * 8),
                ("dense_bytes", C.c_uint64), ("expert_bytes", C.c_uint64), ("slab_bytes_max", C.c_uint64),
                ("params_total", C.c_double), ("params_active", C.c_double), ("cache_slots", C.c_int),
                ("isa", C.c_int), ("n_threads", C.c_int), ("n_io_threads", C.c_int)]


_libs = {}


def load(path):
    if path not in _libs:
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built (make -C oracle with the reference checkout)")
        L = C.CDLL(path)
        L.hearth_default_options.argtypes = [C.POINTER(HearthOptions)]
        L.hearth_open.restype = C.c_void_p
        L.hearth_open.argtypes = [C.POINTER(HearthOptions), C.c_char_p, C.c_size_t]
        L.hearth_close.argtypes = [C.c_void_p]
        L.hearth_eval.restype = C.c_int
        L.hearth_eval.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        L.hearth_info.argtypes = [C.c_void_p, C.POINTER(HearthModelInfo)]
        L.hearth_trace_start.argtypes = [C.c_void_p, C.c_char_p]
        L.hearth_trace_stop.argtypes = [C.c_void_p]
        L.hearth_route_replay.argtypes = [C.c_void_p, C.c_char_p]
        _libs[path] = L
    return _libs[path]


class Engine:
    """One hearth_open handle of a library build (the unchanged reference, or the one with the binding)."""

    def __init__(self, lib_path, model=FIXTURE, threads=2, max_batch=0):
        self.L = load(lib_path)
        o = HearthOptions()
        self.L.hearth_default_options(C.byref(o))
        self._path = os.fsencode(model)
        o.model_path = self._path
        o.cache_gb = 0.05
        o.n_threads = threads
        o.direct_io = 0
        o.max_batch = max_batch
        err = C.create_string_buffer(1024)
        self.h = self.L.hearth_open(C.byref(o), err, 1024)
        if not self.h:
            raise RuntimeError("hearth_open failed: " + err.value.decode())
        info = HearthModelInfo()
        self.L.hearth_info(self.h, C.byref(info))
        self.V = info.vocab_size

    def eval(self, tokens, all_logits=False):
        """(return code, logits [n, V] or [V])."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.full((t.size if all_logits else 1) * self.V, np.nan, np.float32)
        rc = self.L.hearth_eval(self.h, t.ctypes.data, t.size, out.ctypes.data, 1 if all_logits else 0)
        return rc, (out.reshape(t.size, self.V) if all_logits else out)

    def trace_start(self, path):
        return self.L.hearth_trace_start(self.h, os.fsencode(path))

    def trace_stop(self):
        return self.L.hearth_trace_stop(self.h)

    def route_replay(self, path):
        return self.L.hearth_route_replay(self.h, os.fsencode(path))

    def close(self):
        if self.h:
            self.L.hearth_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def session(engine, prompt, steps, trace_path=None):
    """A prompt (all logits) followed by greedy single-token decode steps; returns every logit row."""
    if trace_path:
        assert engine.trace_start(trace_path) == 0
    rc, first = engine.eval(prompt, all_logits=True)
    assert rc == 0, rc
    rows = [first]
    tok = int(np.argmax(first[-1]))
    for _ in range(steps):
        rc, lg = engine.eval([tok])
        assert rc == 0, rc
        rows.append(lg[None, :])
        tok = int(np.argmax(lg))
    if trace_path:
        assert engine.trace_stop() == 0
    return np.concatenate(rows)
