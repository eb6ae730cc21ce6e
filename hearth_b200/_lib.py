"""ctypes binding of include/hearth_b200.h (the in-tree libhearth_b200.so).

There is no fallback: if the CUDA library is missing or cannot load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhearth_b200.so")

# dtypes, engine/include/hearth.h:40-43
F32, F16, BF16, Q8, Q4 = 0, 1, 2, 3, 4
POLICY_LRU, POLICY_LFU = 0, 1
SCORE_SOFTMAX, SCORE_SIGMOID = 0, 1

HXB_OK, HXB_E_ARG, HXB_E_TOKEN, HXB_E_CAPACITY, HXB_E_IO, HXB_E_NOMEM, HXB_E_FORMAT, HXB_E_DEVICE, \
    HXB_E_UNSUPPORTED = 0, -1, -2, -3, -4, -5, -6, -7, -8

# every symbol the header declares (checked by the CPU tests)
EXPORTS = [
    "hxb_version", "hxb_last_error", "hxb_device_count", "hxb_row_bytes", "hxb_matmul", "hxb_dequantize",
    "hxb_act_quantize_dev", "hxb_matmul_dev", "hxb_dequantize_dev", "hxb_expf_dev",
    "hxb_moe_default_config", "hxb_moe_open", "hxb_moe_close", "hxb_moe_set_layer", "hxb_moe_set_expert",
    "hxb_moe_synthesize", "hxb_moe_slab_bytes", "hxb_moe_forward", "hxb_moe_forward_dev", "hxb_moe_forward_routed", "hxb_moe_ep_ipc_handle", "hxb_moe_ep_connect", "hxb_moe_layer",
    "hxb_moe_layer_dev", "hxb_moe_last_routing", "hxb_moe_get_stats", "hxb_moe_reset_stats",
    "hxb_moe_is_resident", "hxb_moe_tick", "hxb_moe_prefetch", "hxb_moe_seed_heat", "hxb_moe_set_copy_hook",
    "hxb_moe_sync", "hxb_moe_profile", "hxb_matmul_noalloc", "hxb_moe_phase_trace", "hxb_moe_decode_path",
    "hxb_moe_ep_layer_dev", "hxb_moe_ep_combine_dev", "hxb_container_probe", "hxb_moe_load_container",
    "hxb_moe_share_expert", "hxb_model_default_options", "hxb_model_open", "hxb_model_close", "hxb_model_info",
    "hxb_model_forward", "hxb_model_last_routes", "hxb_model_set_replay", "hxb_model_moe", "hxb_model_synthesize",
    "hxb_model_forward_dev", "hxb_model_sync", "hxb_moe_get_expert",
]


class MoeConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("expert_ffn_dim", C.c_int), ("n_experts", C.c_int),
                ("top_k", C.c_int), ("score_fn", C.c_int), ("score_bias", C.c_int), ("n_group", C.c_int),
                ("topk_group", C.c_int), ("norm_topk_prob", C.c_int), ("routed_scale", C.c_float),
                ("residual_scale", C.c_float), ("norm_eps", C.c_float), ("expert_dtype", C.c_int),
                ("shared_ffn_dim", C.c_int), ("shared_dtype", C.c_int), ("shared_gate", C.c_int),
                ("max_tokens", C.c_int), ("cache_gb", C.c_double), ("policy", C.c_int), ("heat_decay", C.c_float),
                ("device", C.c_int), ("ep_size", C.c_int), ("ep_rank", C.c_int), ("prefetch_next", C.c_int)]


class ModelOptions(C.Structure):
    _fields_ = [("device", C.c_int), ("max_batch", C.c_int), ("max_seq", C.c_int), ("cache_gb", C.c_double),
                ("policy", C.c_int)]


class ModelArch(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("qk_norm", C.c_int), ("rope_theta", C.c_float), ("dense_dtype", C.c_int), ("sigma_dense", C.c_float),
                ("moe", MoeConfig)]


class ContainerInfo(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_moe_layers", C.c_int), ("n_expert_entries", C.c_int),
                ("n_physical_slabs", C.c_int), ("n_aliased", C.c_int), ("expert_dtype", C.c_int),
                ("slab_bytes", C.c_uint64)]


class MoeStats(C.Structure):
    _fields_ = [("tokens", C.c_uint64), ("forward_calls", C.c_uint64), ("expert_uses", C.c_uint64),
                ("expert_loads_unique", C.c_uint64), ("hits", C.c_uint64), ("misses", C.c_uint64),
                ("evictions", C.c_uint64), ("prefetch_issued", C.c_uint64), ("prefetch_used", C.c_uint64),
                ("prefetch_wasted", C.c_uint64), ("bytes_copied", C.c_uint64), ("copies", C.c_uint64),
                ("copy_errors", C.c_uint64), ("n_slots", C.c_int), ("resident", C.c_int), ("pinned", C.c_int),
                ("slot_bytes", C.c_uint64), ("wall_s", C.c_double), ("stall_s", C.c_double),
                ("host_bytes", C.c_uint64)]


COPY_HOOK = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int)

_lib = None


def lib() -> C.CDLL:
    """Loads libhearth_b200.so, building it first if it is absent (nvcc, sm_100a)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _b
        _b.build()
    L = C.CDLL(LIB_PATH)
    vp, i, i64, sz, f = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
    sig = {
        "hxb_version": (C.c_char_p, []), "hxb_last_error": (C.c_char_p, []), "hxb_device_count": (i, []),
        "hxb_row_bytes": (sz, [i, i64]),
        "hxb_matmul": (i, [i, vp, i64, i64, vp, i, vp]),
        "hxb_dequantize": (i, [i, vp, i64, i64, vp]),
        "hxb_act_quantize_dev": (i, [vp, i64, i, vp, vp]),
        "hxb_matmul_dev": (i, [i, vp, i64, vp, i, vp, i64, i64, i64, vp]),
        "hxb_dequantize_dev": (i, [i, vp, i64, i64, vp, vp]),
        "hxb_expf_dev": (i, [C.c_uint32, i64, vp, vp]),
        "hxb_moe_default_config": (None, [C.POINTER(MoeConfig)]),
        "hxb_moe_open": (vp, [C.POINTER(MoeConfig), C.c_char_p, sz]),
        "hxb_moe_close": (None, [vp]),
        "hxb_moe_set_layer": (i, [vp, i, vp, vp, vp, vp, vp, vp, vp]),
        "hxb_moe_set_expert": (i, [vp, i, i, vp, sz]),
        "hxb_moe_synthesize": (i, [vp, C.c_uint64, f, f]),
        "hxb_moe_slab_bytes": (sz, [vp]),
        "hxb_moe_forward": (i, [vp, vp, i, i, i]),
        "hxb_moe_forward_dev": (i, [vp, vp, i, i, i, vp]),
        "hxb_moe_forward_routed": (i, [vp, vp, i, i, i, vp]),
        "hxb_moe_ep_ipc_handle": (i, [vp, vp]),
        "hxb_moe_ep_connect": (i, [vp, vp]),
        "hxb_moe_layer": (i, [vp, i, vp, i, vp]),
        "hxb_moe_layer_dev": (i, [vp, i, vp, i, vp, vp]),
        "hxb_moe_last_routing": (i, [vp, vp, vp, i]),
        "hxb_moe_get_stats": (i, [vp, C.POINTER(MoeStats)]),
        "hxb_moe_reset_stats": (None, [vp]),
        "hxb_moe_is_resident": (i, [vp, i, i]),
        "hxb_moe_tick": (None, [vp]),
        "hxb_moe_prefetch": (i, [vp, i, vp, i]),
        "hxb_moe_seed_heat": (i, [vp, vp, i, f, i]),
        "hxb_moe_set_copy_hook": (None, [vp, COPY_HOOK, vp]),
        "hxb_moe_sync": (i, [vp, vp]),
        "hxb_moe_profile": (i, [vp, i, i, C.POINTER(C.c_double)]),
        "hxb_matmul_noalloc": (i, [i, vp, i64, i64, vp, i, vp, vp]),
        "hxb_moe_phase_trace": (i64, [vp, vp, i64]),
        "hxb_moe_decode_path": (C.c_int, [vp]),
        "hxb_moe_ep_layer_dev": (i, [vp, i, vp, i, vp, vp]),
        "hxb_moe_ep_combine_dev": (i, [vp, i, vp, i, vp, vp]),
        "hxb_container_probe": (i, [C.c_char_p, C.POINTER(MoeConfig), C.POINTER(ContainerInfo), C.c_char_p, sz]),
        "hxb_moe_load_container": (i, [vp, C.c_char_p]),
        "hxb_moe_share_expert": (i, [vp, i, i, i, i]),
        "hxb_model_default_options": (None, [C.POINTER(ModelOptions)]),
        "hxb_model_open": (vp, [C.c_char_p, C.POINTER(ModelOptions), C.c_char_p, sz]),
        "hxb_model_close": (None, [vp]),
        "hxb_model_info": (i, [vp, vp, vp, vp, vp, vp, vp]),
        "hxb_model_forward": (i, [vp, vp, i, i, vp, i]),
        "hxb_model_last_routes": (i, [vp, vp, i]),
        "hxb_model_set_replay": (i, [vp, vp, i]),
        "hxb_model_moe": (vp, [vp]),
        "hxb_model_forward_dev": (i, [vp, vp, i, i, vp, i, vp]),
        "hxb_model_sync": (i, [vp, vp]),
        "hxb_moe_get_expert": (i, [vp, i, i, vp, sz]),
        "hxb_model_synthesize": (vp, [C.POINTER(ModelArch), C.POINTER(ModelOptions), C.c_uint64, C.c_char_p, sz]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return (lib().hxb_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with {rc}: {last_error()}")
