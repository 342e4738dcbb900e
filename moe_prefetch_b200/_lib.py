"""ctypes binding of libmoeb200.so (the C ABI in include/moeb200.h).

The library is built in-tree (``python -m moe_prefetch_b200.build``).  There is
no fallback: if the shared object is missing or fails to load, every entry
point raises -- the product path never silently runs on the CPU.
"""
import ctypes as C
import os

from .build import LIB

MOE_OK = 0
ERRORS = {
    -1: "MOE_ERR_ARG", -2: "MOE_ERR_CUDA", -3: "MOE_ERR_OOM", -4: "MOE_ERR_UNSUPPORTED",
    -5: "MOE_ERR_TIMEOUT", -6: "MOE_ERR_STATE", -7: "MOE_ERR_DEVICE",
}
QTYPE_Q4_K = 12
QTYPE_Q6_K = 14
STAT_NAMES = ["steps", "clock", "hits", "misses", "uploads", "scheduled", "copied",
              "published", "admit_ok", "admit_denied", "table_flushes", "upload_bytes", "upload_ns"]
# moe_stream_stats, in the C ABI's order
STREAM_STAT_NAMES = ["lookaheads", "offered", "chunks", "bytes", "words", "dropped_late",
                     "dropped_posted", "given_back", "in_time", "late"]


class MoeError(RuntimeError):
    def __init__(self, code, msg=""):
        self.code = code
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")


class MoeCfg(C.Structure):
    """struct moe_cfg (include/moeb200.h)."""
    _fields_ = [
        ("n_layers", C.c_int32), ("n_expert", C.c_int32), ("n_used", C.c_int32),
        ("n_embd", C.c_int32), ("n_ff", C.c_int32), ("down_type", C.c_int32),
        ("n_slots", C.c_int32), ("slot_profile", C.c_void_p), ("max_inserts", C.c_int32),
        ("admit_mode", C.c_int32), ("admit_window", C.c_int32), ("admit_half", C.c_int32),
        ("admit_floor", C.c_float), ("spec_probation", C.c_int32),
        ("batch_tables", C.c_int32), ("cache_prior", C.c_float), ("early_issue", C.c_int32),
        ("freeze", C.c_int32), ("use_heat_counts", C.c_int32), ("device", C.c_int32),
        ("n_shared", C.c_int32), ("predict_top", C.c_int32),
        ("stream", C.c_int32), ("stream_per_layer", C.c_int32), ("stream_reserve", C.c_int32),
        ("stream_gbps", C.c_float), ("stream_topk", C.c_int32),
    ]


# host callbacks of include/moeb200.h
OBSERVE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.POINTER(C.c_int32), C.c_int, C.c_int)
PREDICT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_int32), C.c_int,
                         C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_int32), C.c_int)


class MoeLayerInfo(C.Structure):
    _fields_ = [("gate_c", C.c_void_p), ("up_c", C.c_void_p), ("down_c", C.c_void_p),
                ("dev_table", C.c_void_p), ("gate_bytes", C.c_int64),
                ("down_bytes", C.c_int64), ("n_slots", C.c_int32), ("il", C.c_int32)]


class MoeDecodeDbg(C.Structure):
    _fields_ = [("x", C.c_void_p), ("ids", C.c_void_p), ("w", C.c_void_p), ("y", C.c_void_p),
                ("prof", C.c_void_p), ("starve", C.c_int32), ("spec", C.c_int32)]


P = C.c_void_p
I = C.c_int
I64 = C.c_int64
F = C.c_float

# name -> (restype, argtypes); the exported surface of include/moeb200.h
SIGNATURES = {
    "moe_create": (I, [P, P]),
    "moe_destroy": (None, [P]),
    "moe_last_error": (C.c_char_p, [P]),
    "moe_get_layer": (I, [P, I, P]),
    "moe_set_router": (I, [P, I, P]),
    "moe_set_expert_weights": (I, [P, I, P, P, P]),
    "moe_place": (I, [P, I, P, I]),
    "moe_set_shared_expert": (I, [P, I, P, P, P]),
    "moe_layer_forward": (I, [P, I, P, P, I, P, P, P]),
    "moe_layer_forward_noalloc": (I, [P, I, P, P, I, P, P, P]),
    "moe_layer_forward_path": (I, [P, I, P, P, I, P, P, I, P]),
    "moe_ep_route_pack": (I, [P, I, P, I, I, I, P, P, P, P, P, P, P]),
    "moe_experts_rows": (I, [P, I, P, P, I, P, I, P]),
    "moe_ep_combine": (I, [P, P, P, P, I, P, P, P]),
    "moe_set_observe_hook": (I, [P, P, P]),
    "moe_set_predictor": (I, [P, P, P]),
    "moe_ep_mailbox_create": (I, [P, I, I, I, P]),
    "moe_ep_mailbox_connect": (I, [P, P]),
    "moe_ep_push": (I, [P, I, P, P, P, P]),
    "moe_ep_serve": (I, [P, I, I, I, P]),
    "moe_ep_collect": (I, [P, P, P, I, P, P, P]),
    "moe_decode": (I, [P, P, P, I, P, P]),
    "moe_decode_host": (I, [P, P, P, I, P]),
    "moe_sync": (I, [P, P]),
    "moe_set_wait_limit": (I, [P, C.c_uint64]),
    "moe_decode_info": (I, [P, P, I]),
    "moe_observe": (I, [P, I, P, I, I, P]),
    "moe_step": (I, [P, P]),
    "moe_requires_sync": (I, [P]),
    "moe_get_tables": (I, [P, I, P, P, P, P, P]),
    "moe_get_gate_state": (I, [P, I, P, P, P, P]),
    "moe_get_stats": (I, [P, P, I]),
    "moe_stream_stats": (I, [P, P, I]),
    "moe_set_evictor": (I, [P, I, P, I, P, P, P, P]),
    "moe_warm_start": (I, [P, P]),
    "moe_router_run": (I, [P, P, I, I, I, P, I, F, I, P, P, P, P]),
    "moe_quantize": (I, [P, P, I64, I, P]),
    "moe_synth_weights": (I, [P, I64, I, C.c_uint64, F, P]),
    "moe_synth_f32": (I, [P, I64, C.c_uint64, F, P]),
    "moe_xc_create": (I, [I, I, I, I64, P, I, P]),
    "moe_xc_destroy": (None, [P]),
    "moe_xc_prefetch": (I, [P, I, P, I]),
    "moe_xc_query": (I, [P, I, P, I, P]),
    "moe_xc_admit": (I, [P, I, P, I]),
    "moe_xc_sync": (I, [P]),
    "moe_xc_vram_bytes": (I64, [P]),
    "moe_xc_stats": (I, [P, P]),
    "moe_xc_slab": (P, [P, I]),
    "moe_xc_slot_of": (I, [P, I, I]),
}

_lib = None


def load():
    """Load libmoeb200.so; raise if it is not built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise ImportError(
                f"{LIB} is not built; run `python -m moe_prefetch_b200.build` "
                "(the MoE hot path has no CPU fallback)")
        lib = C.CDLL(LIB)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc, ctx=None, what=""):
    if rc is not None and rc < 0:
        msg = ""
        if ctx:
            m = load().moe_last_error(ctx)
            msg = m.decode() if m else ""
        raise MoeError(rc, f"{what}: {msg}" if what else msg)
    return rc
