"""ctypes binding of libgalactus_b200.so (the C-ABI declared in include/galactus_b200.h).

The library is built in-tree by ``python -m galactus_b200.build``. There is no
fallback: importing this module without the built library raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgalactus_b200.so"

GX_OK = 0
STATUS = {
    0: "GX_OK", -1: "GX_ERR_INVALID", -2: "GX_ERR_TYPE", -3: "GX_ERR_ALIGN", -4: "GX_ERR_DOMAIN",
    -5: "GX_ERR_BATCH", -6: "GX_ERR_SLOTS", -7: "GX_ERR_CUDA", -8: "GX_ERR_TIMEOUT", -9: "GX_ERR_NOMEM",
    -10: "GX_ERR_COPY", -11: "GX_ERR_STATE", -12: "GX_ERR_DEVICE", -13: "GX_ERR_COMM",
}
for _code, _name in STATUS.items():
    globals()[_name] = _code

TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K, TYPE_IQ1_S, TYPE_MXFP4 = 8, 12, 14, 15, 19, 39
POLICY_AUTO, POLICY_UNIFORM, POLICY_PLAN, POLICY_FREQUENCY, POLICY_LRU = range(5)
ACT_SWIGLU, ACT_SWIGLU_OAI = 0, 1

BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q8_K: 292, TYPE_Q4_K: 144, TYPE_Q6_K: 210, TYPE_MXFP4: 17, TYPE_IQ1_S: 50}
BLOCK_ELEMS = {TYPE_Q8_0: 32, TYPE_Q8_K: 256, TYPE_Q4_K: 256, TYPE_Q6_K: 256, TYPE_MXFP4: 32, TYPE_IQ1_S: 256}
TYPE_NAMES = {TYPE_Q8_0: "q8_0", TYPE_Q4_K: "q4_K", TYPE_Q6_K: "q6_K", TYPE_Q8_K: "q8_K",
              TYPE_IQ1_S: "iq1_s", TYPE_MXFP4: "mxfp4"}


def row_bytes(t: int, n: int) -> int:
    return (n // BLOCK_ELEMS[t]) * BLOCK_BYTES[t]


def vec_dot_type(t: int) -> int:
    return TYPE_Q8_0 if t in (TYPE_Q8_0, TYPE_MXFP4) else TYPE_Q8_K


class gx_profile(C.Structure):
    _fields_ = [("first_layer", C.c_uint32), ("last_layer", C.c_uint32), ("experts", C.c_uint32),
                ("used", C.c_uint32), ("record_bytes", C.POINTER(C.c_uint64)),
                ("record_bytes_raw", C.POINTER(C.c_uint64))]


class gx_serve_stats(C.Structure):
    _fields_ = [("hits", C.c_uint32), ("misses", C.c_uint32), ("evictions", C.c_uint32),
                ("distinct", C.c_uint32), ("bytes_copied", C.c_uint64)]


GX_EP_MODULO, GX_EP_BLOCK = 0, 1


class gx_gguf_moe(C.Structure):
    _fields_ = [("arch", C.c_char * 64), ("first_layer", C.c_uint32), ("last_layer", C.c_uint32),
                ("experts", C.c_uint32), ("used", C.c_uint32), ("block_count", C.c_uint32),
                ("type_gate", C.c_uint32), ("type_up", C.c_uint32), ("type_down", C.c_uint32),
                ("hidden", C.c_uint64), ("intermediate", C.c_uint64),
                ("record_bytes", C.c_uint64), ("record_bytes_raw", C.c_uint64)]

GX_PLAN_TIMING = 1
GX_PLAN_LAYERWISE = 2
GX_GATING_SOFTMAX, GX_GATING_SIGMOID, GX_GATING_SOFTMAX_WEIGHT = 0, 1, 2


class gx_router_desc(C.Structure):
    _fields_ = [("gating", C.c_int32), ("n_expert", C.c_int32), ("n_expert_used", C.c_int32),
                ("n_groups", C.c_int32), ("n_group_used", C.c_int32), ("norm_w", C.c_int32),
                ("scale_w", C.c_int32), ("w_scale", C.c_float)]


class gx_stack_plan_info(C.Structure):
    _fields_ = [("stack_kernel", C.c_int32), ("grid", C.c_int32), ("threads", C.c_int32),
                ("ctas_per_sm", C.c_int32), ("stages", C.c_int32), ("rows_gate_up", C.c_int32),
                ("rows_down", C.c_int32), ("smem_bytes", C.c_uint32), ("tensor_cores", C.c_int32)]


class gx_arena_config(C.Structure):
    _fields_ = [("profile", gx_profile), ("capacity_bytes", C.c_uint64), ("protected_fraction", C.c_double),
                ("policy", C.c_int), ("plan_quotas", C.POINTER(C.c_uint32)), ("device", C.c_int),
                ("host_tier", C.c_int), ("max_tokens", C.c_int64), ("hidden", C.c_int64),
                ("intermediate", C.c_int64), ("host_tier_base", C.c_void_p)]


class gx_arena_stats(C.Structure):
    _fields_ = [("serves", C.c_uint64), ("hits", C.c_uint64), ("misses", C.c_uint64),
                ("evictions", C.c_uint64), ("bytes_h2d", C.c_uint64), ("copies", C.c_uint64)]


class gx_layer_desc(C.Structure):
    _fields_ = [("type_gate", C.c_int32), ("type_up", C.c_int32), ("type_down", C.c_int32), ("act", C.c_int32),
                ("alpha", C.c_float), ("limit", C.c_float), ("hidden", C.c_int64), ("intermediate", C.c_int64),
                ("off_gate", C.c_uint64), ("off_up", C.c_uint64)]


class gx_shared_expert(C.Structure):
    _fields_ = [("record", C.c_void_p), ("desc", gx_layer_desc)]


_P = C.c_void_p
_I64 = C.c_int64
_SIGS = {
    "gx_status_string": (C.c_char_p, [C.c_int]),
    "gx_version": (C.c_char_p, []),
    "gx_device_init": (C.c_int, [C.c_int]),
    "gx_device_error": (C.c_int, [C.POINTER(C.c_int32)]),
    "gx_policy_create": (C.c_int, [C.POINTER(gx_profile), C.c_uint64, C.c_double, C.c_int, C.POINTER(C.c_uint32),
                                   C.POINTER(_P)]),
    "gx_policy_destroy": (None, [_P]),
    "gx_policy_quota": (C.c_int, [_P, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                  C.POINTER(C.c_uint32)]),
    "gx_policy_serve": (C.c_int, [_P, C.c_uint32, C.POINTER(C.c_int32), C.c_uint32, C.POINTER(C.c_int32),
                                  C.POINTER(C.c_uint8), C.POINTER(C.c_int32), C.POINTER(gx_serve_stats)]),
    "gx_policy_slot_of": (C.c_int32, [_P, C.c_uint32, C.c_uint32]),
    "gx_policy_counters": (C.c_int, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "gx_arena_create": (C.c_int, [C.POINTER(gx_arena_config), C.POINTER(_P)]),
    "gx_arena_destroy": (C.c_int, [_P]),
    "gx_arena_host_record": (_P, [_P, C.c_uint32, C.c_uint32]),
    "gx_load_record": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_uint64]),
    "gx_arena_layer_view": (C.c_int, [_P, C.c_uint32, C.POINTER(_P), C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)]),
    "gx_arena_policy": (_P, [_P]),
    "gx_remap_serve": (C.c_int, [_P, C.c_uint32, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P,
                                 C.POINTER(gx_serve_stats)]),
    "gx_arena_read_slot": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_uint64]),
    "gx_arena_warm_all": (C.c_int, [_P, _P]),
    "gx_stats": (C.c_int, [_P, C.POINTER(gx_arena_stats)]),
    "gx_arena_timing": (C.c_int, [_P, C.c_int]),
    "gx_arena_timing_read": (C.c_int, [_P, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "gx_mul_mat_id": (C.c_int, [C.c_int, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64,
                                _I64, _I64, _P, _P]),
    "gx_quantize_rows": (C.c_int, [C.c_int, _P, _I64, _I64, _I64, _P, _I64, _P]),
    "gx_swiglu": (C.c_int, [_P, _P, _P, _I64, _P]),
    "gx_swiglu_oai": (C.c_int, [_P, _P, _P, _I64, C.c_float, C.c_float, _P]),
    "gx_combine": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "gx_expf": (C.c_int, [_P, _P, _I64, _P]),
    "gx_moe_layer_forward": (C.c_int, [_P, C.c_uint32, C.POINTER(gx_layer_desc), _P, _P, _P, _I64, _I64, _P, _P,
                                       C.POINTER(gx_serve_stats)]),
    "gx_moe_layer_forward_shared": (C.c_int, [_P, C.c_uint32, C.POINTER(gx_layer_desc), _P, _P, _P, _I64, _I64,
                                             C.POINTER(gx_shared_expert), _P, _P, C.POINTER(gx_serve_stats)]),
    "gx_moe_stack_forward": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(gx_layer_desc), C.POINTER(_P), _P,
                                       C.POINTER(_P), _I64, _I64, C.POINTER(_P), _P, C.POINTER(gx_serve_stats)]),
    "gx_stack_plan_create": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(gx_layer_desc), C.POINTER(_P),
                                       C.POINTER(_P), C.POINTER(_P), _I64, _I64, C.c_int, C.POINTER(_P)]),
    "gx_stack_plan_run": (C.c_int, [_P, _P, _P, C.POINTER(gx_serve_stats)]),
    "gx_stack_plan_timing": (C.c_int, [_P, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "gx_stack_plan_info_get": (C.c_int, [_P, C.POINTER(gx_stack_plan_info)]),
    "gx_stack_plan_destroy": (C.c_int, [_P]),
    "gx_stack_plan_run_routed": (C.c_int, [_P, C.POINTER(gx_router_desc), _P, _I64, _P, _P, _P,
                                           C.POINTER(gx_serve_stats)]),
    "gx_router_forward": (C.c_int, [C.POINTER(gx_router_desc), _P, _I64, _P, _I64, _I64, _P, _P, _P, _P, _P]),
    "gx_arena_slot_table": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_int, _P]),
    "gx_gguf_moe_info": (C.c_int, [C.c_char_p, _P]),
    "gx_arena_load_gguf": (C.c_int, [_P, C.c_char_p, _P]),
    "gx_fnv1a64": (C.c_uint64, [_P, C.c_uint64]),
    "gx_route_observer_open": (C.c_int, [C.c_char_p, C.c_char_p, C.c_uint64]),
    "gx_route_observer_close": (C.c_int, []),
    "gx_cache_plan_load": (C.c_int, [C.c_char_p, C.POINTER(_P)]),
    "gx_cache_plan_destroy": (None, [_P]),
    "gx_cache_plan_info": (C.c_int, [_P, _P, _P, _P, _P, C.c_char_p, C.c_size_t]),
    "gx_cache_plan_curve": (C.c_int, [_P, C.c_uint32, _P]),
    "gx_plan_layer_quotas": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.c_uint32, C.c_uint32, _P]),
    "gx_policy_plan_quotas": (C.c_int, [C.POINTER(gx_profile), C.c_uint64, C.c_double, _P, _P]),
    "gx_ep_owner": (C.c_int, [C.c_int32, C.c_uint32, C.c_int32, C.c_int32, _P, _P]),
    "gx_ep_plan": (C.c_int, [C.c_int32, C.c_uint32, C.c_int32, _P, _I64, _I64, _P, _P]),
    "gx_ep_init": (C.c_int, [_P, _P, C.c_int32, C.c_int32, C.c_uint32, C.c_int32, C.POINTER(_P)]),
    "gx_ep_destroy": (C.c_int, [_P]),
    "gx_ep_dispatch": (C.c_int, [_P, C.c_uint32, _P, _P, _I64, _I64, _I64, _P]),
    "gx_ep_compute": (C.c_int, [_P, C.POINTER(gx_layer_desc), _P, C.POINTER(gx_serve_stats)]),
    "gx_ep_combine": (C.c_int, [_P, _P, _P, _P]),
    "gx_ep_layer_forward": (C.c_int, [_P, C.c_uint32, C.POINTER(gx_layer_desc), _P, _P, _P, _I64, _I64, _P, _P,
                                      C.POINTER(gx_serve_stats)]),
    "gx_ep_stack_forward": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(gx_layer_desc), C.POINTER(_P), _P,
                                     C.POINTER(_P), _I64, _I64, C.POINTER(_P), _P, C.POINTER(gx_serve_stats)]),
    "gx_moe_ffn_noalloc": (C.c_int, [C.POINTER(gx_layer_desc), _P, C.c_uint64, C.c_uint32, _P, _P, _P, _I64, _I64,
                                     _P, _P]),
    "gx_synth_normal": (C.c_int, [_P, _I64, C.c_uint64, C.c_uint64, C.c_float, _P]),
    "gx_synth_weights": (C.c_int, [C.c_int, _P, _I64, _I64, C.c_uint64, C.c_uint64, C.c_float, _P]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library. Raises if it was not built: there is no fallback path."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m galactus_b200.build`")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def declared_symbols() -> list[str]:
    return list(_SIGS)


class GxError(RuntimeError):
    def __init__(self, code: int, where: str = ""):
        self.code = code
        msg = lib().gx_status_string(code).decode()
        super().__init__(f"{where}: {STATUS.get(code, code)} ({msg})")


def check(code: int, where: str = "") -> None:
    if code != GX_OK:
        raise GxError(code, where)
