"""ctypes binding of oracle/liboracle.so (moe_oracle.c) -- TEST INFRASTRUCTURE.

Each function states the reference code it restates; the C source carries
the file:line citations.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PRED_PATH = os.path.join(HERE, "_ref", "libref_predictor.so")


def reference_dir():
    """Where the reference project's tree is read from (test set-up only):
    $MOE_REFERENCE_DIR, else a `reference` directory beside this repository."""
    return os.environ.get("MOE_REFERENCE_DIR") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")

QTYPE_Q4_K = 12
QTYPE_Q6_K = 14
Q4K_BYTES = 144
Q6K_BYTES = 210
QK_K = 256


def build(force=False):
    """Compile liboracle.so (and the reference predictor when the reference
    tree is present) with oracle/Makefile."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.check_call(["make", "-s", "-C", HERE])
    ref = reference_dir()
    if os.path.isdir(os.path.join(ref, "cpp")) and (force or not os.path.exists(REF_PRED_PATH)):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", "REF=" + ref])


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float


def _declare(L):
    L.or_f32_to_f16.argtypes = [F32]
    L.or_f32_to_f16.restype = C.c_uint16
    L.or_f16_to_f32.argtypes = [C.c_uint16]
    L.or_f16_to_f32.restype = F32
    L.or_expf.argtypes = [F32]
    L.or_expf.restype = F32
    for n in ("or_quantize_q4_K", "or_quantize_q6_K", "or_dequantize_q4_K",
              "or_dequantize_q6_K", "or_q8_K_roundtrip"):
        getattr(L, n).argtypes = [P, P, I64]
        getattr(L, n).restype = None
    L.or_quantize_q8_1.argtypes = [P, P, P, P, I64]
    L.or_dot_q4_K_q8_1.argtypes = [P, P, P, P, I64]
    L.or_dot_q4_K_q8_1.restype = C.c_double
    L.or_dot_q6_K_q8_1.argtypes = [P, P, P, P, I64]
    L.or_dot_q6_K_q8_1.restype = C.c_double
    L.or_combine_f32.argtypes = [P, P, C.c_int, C.c_int, P]
    L.or_combine_f32.restype = None
    for n in ("or_dot_q4_K_q8_1_f32", "or_dot_q6_K_q8_1_f32"):
        getattr(L, n).argtypes = [P, P, P, P, I64]
        getattr(L, n).restype = F32
    L.or_router.argtypes = [P, P, C.c_int, C.c_int, P, C.c_int, P, P, P, P]
    L.or_router_select.argtypes = [P, C.c_int, P, C.c_int, P, P, P]
    L.or_router_fused.argtypes = [P, P, C.c_int, C.c_int, P, P, C.c_int, F32, P, C.c_int, P, P,
                                  P, P]
    L.or_router_dot.argtypes = [P, P, C.c_int]
    L.or_router_dot.restype = F32
    L.or_expert_row.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, P, P, P]
    L.or_expert_row_q8K.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, P, P]
    layer_args = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P, P,
                  C.c_int, P, P, P, C.c_int]
    L.or_moe_layer.argtypes = layer_args
    L.or_moe_experts_f32.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P,
                                     P, C.c_int, P, C.c_int]
    L.or_moe_experts_f32.restype = None
    L.or_moe_experts.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P, P, C.c_int,
                                 P, C.c_int]
    L.or_moe_layer_q8K.argtypes = layer_args
    L.or_moe_layer_cpu_fast.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P,
                                        P, C.c_int, P, P, P, C.c_int]
    L.or_cache_create.argtypes = [P]
    L.or_cache_create.restype = P
    L.or_cache_destroy.argtypes = [P]
    L.or_cache_observe.argtypes = [P, C.c_int, P, C.c_int, C.c_int, C.c_int]
    L.or_cache_step.argtypes = [P]
    L.or_cache_n_slots.argtypes = [P, C.c_int]
    L.or_cache_n_slots.restype = I32
    L.or_cache_tables.argtypes = [P, C.c_int, P, P, P, P, P]
    L.or_cache_dev_table.argtypes = [P, C.c_int, P, P]
    L.or_cache_stats.argtypes = [P, P]
    L.or_cache_jobs.argtypes = [P, P, C.c_int]
    L.or_cache_jobs.restype = C.c_int
    L.or_cache_gate_state.argtypes = [P, C.c_int, P, P, P, P]
    L.or_cache_map_header.argtypes = [P, C.c_char_p, C.c_int]
    L.or_cache_map_header.restype = C.c_int
    L.or_cache_map_frame.argtypes = [P, C.c_char_p, C.c_int]
    L.or_cache_map_frame.restype = C.c_int
    L.or_cache_save_heat.argtypes = [P, C.c_char_p]
    L.or_cache_save_heat.restype = C.c_int
    L.or_cache_load_heat.argtypes = [P, C.c_char_p]
    L.or_cache_load_heat.restype = I64
    L.or_cache_warm_start.argtypes = [P]
    L.or_cache_warm_start.restype = I64
    L.or_cache_set_predictor.argtypes = [P, P, P]
    L.or_evict_score.argtypes = [P, P, F32, P, C.c_int, P, C.c_int, P, C.c_int, P, C.c_int, P,
                                 C.c_int, P]
    L.or_evict_score.restype = None
    L.or_cache_set_evictor.argtypes = [P, C.c_int, P, C.c_int, P, P, P, P]
    L.or_cache_set_evictor.restype = C.c_int
    L.or_greedy_allocate_bytes.argtypes = [P, P, C.c_int, C.c_int, C.c_int, P, C.c_int, P, P, P]
    L.or_greedy_allocate_bytes.restype = C.c_double


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------------------
# scalar / codecs
# ---------------------------------------------------------------------------
def expf(x):
    return lib().or_expf(float(x))


def f32_to_f16_bits(x):
    return lib().or_f32_to_f16(float(x))


def quantize(x, qtype):
    """float32 [..., n] -> uint8 blocks [..., n/256 * block_bytes]."""
    x = _c(x, np.float32)
    n = x.size
    bb = Q4K_BYTES if qtype == QTYPE_Q4_K else Q6K_BYTES
    out = np.empty(n // QK_K * bb, dtype=np.uint8)
    fn = lib().or_quantize_q4_K if qtype == QTYPE_Q4_K else lib().or_quantize_q6_K
    fn(_p(x), _p(out), n)
    return out.reshape(x.shape[:-1] + (x.shape[-1] // QK_K * bb,))


def dequantize(y, qtype, n):
    y = _c(y, np.uint8)
    out = np.empty(n, dtype=np.float32)
    fn = lib().or_dequantize_q4_K if qtype == QTYPE_Q4_K else lib().or_dequantize_q6_K
    fn(_p(y), _p(out), n)
    return out


def quantize_q8_1(x):
    x = _c(x, np.float32).ravel()
    n = x.size
    q = np.empty(n, dtype=np.int8)
    d = np.empty(n // 32, dtype=np.float32)
    s = np.empty(n // 32, dtype=np.float32)
    lib().or_quantize_q8_1(_p(x), _p(q), _p(d), _p(s), n)
    return q, d, s


def q8_K_roundtrip(x):
    x = _c(x, np.float32).ravel()
    out = np.empty_like(x)
    lib().or_q8_K_roundtrip(_p(x), _p(out), x.size)
    return out


def combine_rows(w, rows):
    """The kernels' combine: w [n_tok, k], rows [n_tok, k, n_embd] -> y
    [n_tok, n_embd], per element an fp32 fma chain from 0 in rank order."""
    w = _c(w, np.float32)
    rows = _c(rows, np.float32)
    n_tok, k, n = rows.shape
    y = np.empty((n_tok, n), np.float32)
    for t in range(n_tok):
        lib().or_combine_f32(_p(w[t]), _p(rows[t]), k, n, _p(y[t]))
    return y


def dot_q8_1(row, qtype, q, d, s, order="f64"):
    """One quantised row with Q8_1 activations: "f64" accumulates in double
    (the precision reference), "kernel" in the GPU GEMV kernels' fp32 order."""
    row = _c(row, np.uint8)
    if order == "kernel":
        fn = lib().or_dot_q4_K_q8_1_f32 if qtype == QTYPE_Q4_K else lib().or_dot_q6_K_q8_1_f32
    else:
        fn = lib().or_dot_q4_K_q8_1 if qtype == QTYPE_Q4_K else lib().or_dot_q6_K_q8_1
    return fn(_p(row), _p(q), _p(d), _p(s), q.size)


# ---------------------------------------------------------------------------
# router / rows / layer
# ---------------------------------------------------------------------------
def router_dot(w_row, x):
    w_row = _c(w_row, np.float32)
    x = _c(x, np.float32)
    return lib().or_router_dot(_p(w_row), _p(x), x.size)


def router(W, x, k, prior=None):
    """Returns ids int32[k], weights f32[k], probs f32[E], logits f32[E]."""
    W = _c(W, np.float32)
    x = _c(x, np.float32)
    E, H = W.shape
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    probs = np.empty(E, np.float32)
    logits = np.empty(E, np.float32)
    pr = _c(prior, np.float32) if prior is not None else None
    lib().or_router(_p(W), _p(x), E, H, _p(pr) if pr is not None else None, k,
                    _p(ids), _p(w), _p(probs), _p(logits))
    return ids, w, probs, logits


def router_fused(Wt, r, k, h0, h1, eps=1e-6, prior=None):
    """The decode kernel's fused RMSNorm + router.  Wt [n_embd, n_expert];
    h0/h1 the per-CTA row ranges.  Returns ids, w, x (normalised r), logits."""
    Wt = _c(Wt, np.float32)
    r = _c(r, np.float32)
    H, E = Wt.shape
    h0 = _c(h0, np.int32)
    h1 = _c(h1, np.int32)
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    x = np.empty(H, np.float32)
    logits = np.empty(E, np.float32)
    pr = _c(prior, np.float32) if prior is not None else None
    lib().or_router_fused(_p(Wt), _p(r), E, H, _p(h0), _p(h1), len(h0), eps,
                          _p(pr) if pr is not None else None, k, _p(ids), _p(w), _p(x),
                          _p(logits))
    return ids, w, x, logits


def expert_row(gate, up, down, down_type, n_embd, n_ff, x, q8K=False):
    """One expert's unweighted output row f32[n_embd] (and act f32[n_ff])."""
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    x = _c(x, np.float32)
    out = np.empty(n_embd, np.float32)
    if q8K:
        lib().or_expert_row_q8K(_p(gate), _p(up), _p(down), down_type, n_embd, n_ff,
                                _p(x), _p(out))
        return out, None
    act = np.empty(n_ff, np.float32)
    lib().or_expert_row(_p(gate), _p(up), _p(down), down_type, n_embd, n_ff, _p(x),
                        _p(out), _p(act))
    return out, act


def moe_layer(x, router_w, gate, up, down, down_type, n_ff, k, prior=None,
              n_threads=None, path="q8_1"):
    """x f32[n_tok, n_embd]; gate/up/down uint8 [n_expert, ...] -> (ids, w, y)."""
    x = _c(np.atleast_2d(x), np.float32)
    n_tok, n_embd = x.shape
    router_w = _c(router_w, np.float32)
    n_expert = router_w.shape[0]
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    ids = np.empty((n_tok, k), np.int32)
    w = np.empty((n_tok, k), np.float32)
    y = np.empty((n_tok, n_embd), np.float32)
    pr = _c(prior, np.float32) if prior is not None else None
    nt = n_threads or os.cpu_count()
    fn = lib().or_moe_layer if path == "q8_1" else lib().or_moe_layer_q8K
    fn(_p(x), n_tok, n_embd, n_ff, n_expert, k, _p(router_w),
       _p(pr) if pr is not None else None, _p(gate), _p(up), _p(down), down_type,
       _p(ids), _p(w), _p(y), nt)
    return ids, w, y


def moe_experts(x, ids, w, gate, up, down, down_type, n_ff, n_threads=None, path="q8_1"):
    """y [n_tok, n_embd] = sum_i w[t, i] * expert_row(ids[t, i], x[t]).
    path "q8_1": Q8_1 activations (the GEMV kernels' arithmetic); "f32":
    unquantised activations, exact weights, fp64 accumulation (the reference
    of the fp16 tensor-core GEMM)."""
    x = _c(np.atleast_2d(x), np.float32)
    n_tok, n_embd = x.shape
    ids = _c(np.atleast_2d(ids), np.int32)
    w = _c(np.atleast_2d(w), np.float32)
    k = ids.shape[1]
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    y = np.empty((n_tok, n_embd), np.float32)
    if path == "f32":
        lib().or_moe_experts_f32(_p(x), n_tok, n_embd, n_ff, gate.shape[0], k, _p(ids), _p(w),
                                 _p(gate), _p(up), _p(down), down_type, _p(y),
                                 n_threads or os.cpu_count())
        return y
    lib().or_moe_experts(_p(x), n_tok, n_embd, n_ff, k, _p(ids), _p(w), _p(gate), _p(up),
                         _p(down), down_type, _p(y), n_threads or os.cpu_count())
    return y


def moe_layer_cpu_fast(x, router_w, gate, up, down, down_type, n_ff, k, prior=None,
                       n_threads=None):
    """The timed CPU baseline: one token through ggml-order integer dots."""
    x = _c(x, np.float32).ravel()
    router_w = _c(router_w, np.float32)
    n_expert, n_embd = router_w.shape
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    y = np.empty(n_embd, np.float32)
    pr = _c(prior, np.float32) if prior is not None else None
    lib().or_moe_layer_cpu_fast(_p(x), n_embd, n_ff, n_expert, k, _p(router_w),
                                _p(pr) if pr is not None else None, _p(gate), _p(up),
                                _p(down), down_type, _p(ids), _p(w), _p(y),
                                n_threads or os.cpu_count())
    return ids, w, y


# ---------------------------------------------------------------------------
# slot table
# ---------------------------------------------------------------------------
class OrCacheCfg(C.Structure):
    _fields_ = [("n_layers", I32), ("n_expert", I32), ("n_slots", I32),
                ("slot_profile", C.c_void_p), ("max_inserts", I32),
                ("admit_mode", I32), ("admit_window", I32), ("admit_half", I32),
                ("admit_floor", F32), ("spec_probation", I32), ("batch_tables", I32),
                ("cache_prior", F32), ("early_issue", I32), ("predict_top", I32),
                ("have_pred", I32), ("freeze", I32), ("use_heat_counts", I32)]


ST_NAMES = ["steps", "clock", "hits", "misses", "uploads", "scheduled", "copied",
            "published", "admit_ok", "admit_denied", "table_flushes"]

PREDICT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_int32), C.c_int,
                         C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_int32), C.c_int)


class OracleCache:
    """The slot-table state machine of llama-moecache.cpp (patches 0006/0007/0008),
    deterministic publication."""

    def __init__(self, n_layers, n_expert, n_slots, slot_profile=None, max_inserts=2,
                 admit_mode=0, admit_window=8, admit_half=64, admit_floor=1.0,
                 spec_probation=False, batch_tables=True, cache_prior=0.0,
                 early_issue=False, predict_top=3, predictor=None, freeze=False,
                 use_heat_counts=False):
        self.n_layers, self.n_expert = n_layers, n_expert
        self._profile = (np.ascontiguousarray(slot_profile, np.int32)
                         if slot_profile is not None else None)
        cfg = OrCacheCfg(n_layers, n_expert, n_slots,
                         _p(self._profile) if self._profile is not None else None,
                         max_inserts, admit_mode, admit_window, admit_half, admit_floor,
                         int(spec_probation), int(batch_tables), cache_prior,
                         int(early_issue), predict_top, int(predictor is not None),
                         int(freeze), int(use_heat_counts))
        self.h = lib().or_cache_create(C.byref(cfg))
        self._pred_cb = None
        if predictor is not None:
            def cb(ud, layer, cur, n_cur, nprev, n_nprev, out, k):
                got = predictor(layer, [cur[i] for i in range(n_cur)],
                                [nprev[i] for i in range(n_nprev)], k)
                got = list(got)[:k]
                for i, v in enumerate(got):
                    out[i] = int(v)
                return len(got)
            self._pred_cb = PREDICT_FN(cb)
            lib().or_cache_set_predictor(self.h, C.cast(self._pred_cb, C.c_void_p), None)

    def close(self):
        if self.h:
            lib().or_cache_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def observe(self, layer, ids, force=False):
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        lib().or_cache_observe(self.h, layer, _p(ids), ids.shape[0], ids.shape[1], int(force))

    def step(self):
        lib().or_cache_step(self.h)

    def n_slots(self, layer):
        return lib().or_cache_n_slots(self.h, layer)

    def tables(self, layer):
        ns = self.n_slots(layer)
        es = np.empty(self.n_expert, np.int32)
        se = np.empty(ns, np.int32)
        lu = np.empty(ns, np.uint64)
        fl = np.empty(ns, np.uint8)
        pr = np.empty(ns, np.uint64)
        lib().or_cache_tables(self.h, layer, _p(es), _p(se), _p(lu), _p(fl), _p(pr))
        return {"expert_slot": es, "slot_expert": se, "last_use": lu, "in_flight": fl,
                "protect": pr}

    def dev_table(self, layer):
        t = np.empty(self.n_expert, np.int32)
        p = np.empty(self.n_expert, np.float32)
        lib().or_cache_dev_table(self.h, layer, _p(t), _p(p))
        return t, p

    def stats(self):
        out = np.empty(len(ST_NAMES), np.uint64)
        lib().or_cache_stats(self.h, _p(out))
        return {k: int(v) for k, v in zip(ST_NAMES, out)}

    def jobs(self):
        buf = np.empty((4096, 4), np.int32)
        n = lib().or_cache_jobs(self.h, _p(buf), 4096)
        return buf[:min(n, 4096)].copy()

    def gate_state(self, layer):
        E = self.n_expert
        heat = np.zeros(E, np.float32)
        ml = np.zeros(E, np.uint64)
        mp = np.zeros(E, np.uint64)
        uc = np.zeros(E, np.uint32)
        lib().or_cache_gate_state(self.h, layer, _p(heat), _p(ml), _p(mp), _p(uc))
        return {"heat": heat, "miss_last": ml, "miss_prev": mp, "use_count": uc}

    def map_header(self):
        n = lib().or_cache_map_header(self.h, None, 0)
        buf = C.create_string_buffer(n + 1)
        lib().or_cache_map_header(self.h, buf, n + 1)
        return buf.value.decode()

    def map_frame(self):
        n = lib().or_cache_map_frame(self.h, None, 0)
        buf = C.create_string_buffer(n + 1)
        lib().or_cache_map_frame(self.h, buf, n + 1)
        return buf.value.decode()

    def save_heat(self, path):
        return bool(lib().or_cache_save_heat(self.h, path.encode()))

    def load_heat(self, path):
        return int(lib().or_cache_load_heat(self.h, path.encode()))

    def warm_start(self):
        return int(lib().or_cache_warm_start(self.h))

    def set_evictor(self, model):
        """LLAMA_MOE_EVICTOR: `model` is a MoePredictor (MOEP v3)."""
        arr = evictor_arrays(model, self.n_layers)
        self._ev = arr
        rc = lib().or_cache_set_evictor(self.h, arr["n_model"], _p(arr["layer_of"]), arr["feat_dim"],
                                        _p(arr["off"]), _p(arr["w"]), _p(arr["bias"]), _p(arr["prior"]))
        if rc != 0:
            raise ValueError("or_cache_set_evictor refused the model")


def evictor_arrays(model, n_layers):
    """The arrays an evictor takes (MOEP v3 model of this stack's layers):
    layer_of, off (prev, cur, below, self_prev), w, bias, prior."""
    BLOCK_PREV, BLOCK_CUR, BLOCK_BELOW, BLOCK_SELF_PREV = 1, 2, 3, 4   # MOEP v3 block kinds
    return {"n_model": int(len(model.layer_of)), "feat_dim": int(model.feat_dim),
            "layer_of": np.ascontiguousarray(model.layer_of, np.int32),
            "off": np.array([model.off[BLOCK_PREV], model.off[BLOCK_CUR], model.off[BLOCK_BELOW],
                             model.off[BLOCK_SELF_PREV]], np.int32),
            "w": np.ascontiguousarray(model.w, np.float32),
            "bias": np.ascontiguousarray(model.bias, np.float32),
            "prior": np.ascontiguousarray(model.prior, np.float32)}


def evict_score(model, il, prev=(), cur=(), below=(), self_prev=()):
    """or_evict_score on one layer of a MoePredictor (the C restatement)."""
    arr = evictor_arrays(model, 0)
    m = int(model.index_of[il])
    E = model.n_expert
    lists = [np.ascontiguousarray(x, np.int32) for x in (prev, cur, below, self_prev)]
    out = np.empty(E, np.float32)
    w = np.ascontiguousarray(arr["w"][m])
    b = np.ascontiguousarray(arr["bias"][m])
    lib().or_evict_score(_p(w), _p(b), float(arr["prior"][m]), _p(arr["off"]), E,
                         _p(lists[0]), len(lists[0]), _p(lists[1]), len(lists[1]),
                         _p(lists[2]), len(lists[2]), _p(lists[3]), len(lists[3]), _p(out))
    return out


def greedy_allocate_bytes(per_layer_miss8, grid, n_layers, uniform_cap, frozen_layers,
                          expert_bytes):
    """C restatement of experiments/p7_slot_allocation.py:144-185.
    per_layer_miss8: {grid value: [miss8 per layer]}."""
    miss = np.ascontiguousarray([per_layer_miss8[g] for g in grid], np.float64)
    g = np.ascontiguousarray(grid, np.int32)
    fr = np.ascontiguousarray(sorted(frozen_layers) or [0], np.int32)
    eb = np.ascontiguousarray([b or 0.0 for b in expert_bytes], np.float64)
    cap = np.empty(n_layers, np.int32)
    budget = C.c_double(0.0)
    used = lib().or_greedy_allocate_bytes(_p(miss), _p(g), len(grid), n_layers, uniform_cap,
                                          _p(fr), len(frozen_layers), _p(eb), _p(cap),
                                          C.byref(budget))
    return [int(c) for c in cap], used, budget.value


# ---------------------------------------------------------------------------
# the reference's own predictor (compiled into oracle/_ref)
# ---------------------------------------------------------------------------
class RefPredictor:
    """cpp/moe-predictor.cpp of the reference, through oracle/_ref's shim."""
    _L = None

    @classmethod
    def available(cls):
        return os.path.exists(REF_PRED_PATH)

    @classmethod
    def _lib(cls):
        if cls._L is None:
            L = C.CDLL(REF_PRED_PATH)
            L.refpred_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
            L.refpred_load.restype = P
            L.refpred_free.argtypes = [P]
            L.refpred_info.argtypes = [P, P]
            L.refpred_has_layer.argtypes = [P, C.c_int]
            L.refpred_score.argtypes = [P, C.c_int] + [P, C.c_int] * 4 + [P]
            L.refpred_top_k.argtypes = [P, P, C.c_int, P]
            L.refpred_update.argtypes = [P, C.c_int] + [P, C.c_int] * 5 + [F32]
            L.refpred_update.restype = F32
            L.refpred_save.argtypes = [P, C.c_char_p, C.c_char_p, C.c_int]
            cls._L = L
        return cls._L

    def __init__(self, path):
        err = C.create_string_buffer(512)
        self.h = self._lib().refpred_load(path.encode(), err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        info = np.zeros(10, np.int32)
        self._lib().refpred_info(self.h, _p(info))
        (self.n_expert, self.n_layers, self.feat_dim, self.top_k, self.off_prev,
         self.off_cur, self.off_below, self.off_self_prev, self.off_pca,
         self.n_present) = [int(v) for v in info]

    def has_layer(self, il):
        return bool(self._lib().refpred_has_layer(self.h, il))

    @staticmethod
    def _arr(v):
        a = np.ascontiguousarray(v if v is not None else [], np.int32)
        return a, len(a)

    def score(self, il, prev=None, cur=None, below=None, self_prev=None):
        args = []
        keep = []
        for v in (prev, cur, below, self_prev):
            a, n = self._arr(v)
            keep.append(a)
            args += [_p(a), n]
        out = np.empty(self.n_expert, np.float32)
        self._lib().refpred_score(self.h, il, *args, _p(out))
        return out

    def top_k_ids(self, scores, k):
        scores = _c(scores, np.float32)
        out = np.empty(k, np.int32)
        n = self._lib().refpred_top_k(self.h, _p(scores), k, _p(out))
        return out[:n]

    def update(self, il, truth, lr, prev=None, cur=None, below=None, self_prev=None):
        args = []
        keep = []
        for v in (prev, cur, below, self_prev, truth):
            a, n = self._arr(v)
            keep.append(a)
            args += [_p(a), n]
        return self._lib().refpred_update(self.h, il, *args, lr)

    def save(self, path):
        err = C.create_string_buffer(512)
        ok = self._lib().refpred_save(self.h, path.encode(), err, 512)
        if not ok:
            raise IOError(err.value.decode())

    def close(self):
        if self.h:
            self._lib().refpred_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
