"""MoeStack: the MoE layers of a Qwen3-A3B-class model with a GPU expert slot
cache, driven through the C ABI of libmoeb200.so.

This is the host side of the reference's ``--moe-expert-cache`` path: one
object per device that owns the slot slabs, the device slot table and the
router weights (llama_moe_cache_init, patches/0006:482-763), runs the MoE
layer (build_moe_ffn with the cache chain, patches/0009:659-705) or a whole
batch-1 decode, and advances the cache between tokens (llama_moe_cache_step,
patches/0006:765-953).  PyTorch is used only for device/pinned buffers and
streams; every computation is a CUDA kernel of libmoeb200.so.
"""
import ctypes as C
import sys

import numpy as np
import torch

from . import _lib
from ._lib import MoeCfg, MoeDecodeDbg, MoeError, MoeLayerInfo, QTYPE_Q4_K, QTYPE_Q6_K, STAT_NAMES, STREAM_STAT_NAMES, check
from .config import MoeCacheConfig

Q4K_BYTES, Q6K_BYTES, QK_K = 144, 210, 256


def expert_bytes(n_embd, n_ff, down_type=QTYPE_Q6_K):
    """(gate = up bytes, down bytes) of one expert in ggml block layout."""
    g = n_ff * (n_embd // QK_K) * Q4K_BYTES
    d = n_embd * (n_ff // QK_K) * (Q6K_BYTES if down_type == QTYPE_Q6_K else Q4K_BYTES)
    return g, d


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(C.c_void_p)
    return C.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class _CudaView:
    """A raw device pointer exposed through __cuda_array_interface__, so
    torch.as_tensor can view it without a copy."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


class MoeStack:
    def __init__(self, n_layers, n_expert=128, n_used=8, n_embd=2048, n_ff=768,
                 down_type=QTYPE_Q6_K, cache=None, device=None, n_shared=0):
        self.lib = _lib.load()
        self.cache = cache or MoeCacheConfig()
        self.n_layers, self.n_expert, self.n_used = n_layers, n_expert, n_used
        self.n_embd, self.n_ff, self.down_type = n_embd, n_ff, down_type
        self.n_shared = n_shared
        # default: the caller's current CUDA device (one stack per rank under
        # torch.distributed, each on its own GPU)
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device)
        self.gate_bytes, self.down_bytes = expert_bytes(n_embd, n_ff, down_type)
        self.ns = self.cache.slots_per_layer(n_layers, n_expert)
        self._profile = np.ascontiguousarray(self.ns, np.int32)
        cfg = MoeCfg(n_layers, n_expert, n_used, n_embd, n_ff, down_type,
                     self.cache.n_slots if self.cache.n_slots > 0 else n_expert,
                     self._profile.ctypes.data, self.cache.max_inserts, self.cache.admit_mode,
                     self.cache.admit_window, self.cache.admit_half, self.cache.admit_floor,
                     int(self.cache.spec_probation), int(self.cache.batch_tables),
                     self.cache.cache_prior, int(self.cache.early_issue),
                     int(self.cache.freeze), int(bool(self.cache.heat_file)), device, n_shared,
                     self.cache.predict_top, int(self.cache.stream), self.cache.stream_per_layer,
                     self.cache.stream_reserve, self.cache.stream_gbps, self.cache.stream_topk)
        torch.cuda.set_device(self.device)
        ctx = C.c_void_p()
        check(self.lib.moe_create(C.byref(cfg), C.byref(ctx)), None, "moe_create")
        self.ctx = ctx
        self._host = {}          # keep registered host weights alive
        # the reference's files (LLAMA_MOE_HEAT_FILE / MAP_RECORD / MAP_REPLAY /
        # ROUTE_TRACE): opened at the first forward, decode or step, once the
        # host weights are in (start())
        self._started = False
        self._map_rec = self._map_rep = self._trace = None

    # -- lifetime -------------------------------------------------------------
    def start(self):
        """What llama_moe_cache_init does once the weights exist
        (patches/0007:567-618, 0008:549-571): the heat-file warm start, and
        the map record / replay and route trace files with their header and
        the frame of step 0.  Runs by itself at the first layer_forward,
        decode or step; call it earlier to time it apart."""
        if self._started or not self.ctx:
            return
        self._started = True
        c = self.cache
        if c.evictor:
            # loud either way (patches/0006:521-537): an evictor that silently
            # fails to load looks exactly like one that does not help
            from .predictor import MoePredictor, MoepError
            try:
                m = MoePredictor.load(c.evictor)
                if m.n_expert != self.n_expert:
                    raise MoepError(f"{c.evictor}: {m.n_expert} experts, the stack has {self.n_expert}")
                self.set_evictor(m)
                print(f"moe-cache: evictor loaded, {m.feat_dim} features, {len(m.layer_of)} layers",
                      file=sys.stderr)
            except (OSError, MoepError, MoeError) as e:
                print(f"moe-cache: EVICTOR NOT LOADED: {e}", file=sys.stderr)
        if c.heat_file and self.cache.n_slots > 0:
            counts = load_heat(c.heat_file, self.n_layers, self.n_expert)
            placed = 0
            if counts is not None:
                self.warm_start(counts)
                placed = sum(int((self.tables(il)["slot_expert"] >= 0).sum()) for il in range(self.n_layers))
            # loud either way, as the reference: a missing file is a cold start
            print(f"moe-cache: heat file {c.heat_file}: "
                  f"{0 if counts is None else int((counts > 0).sum())} records, {placed} experts placed before "
                  f"the first token{'' if counts is not None else ' (COLD START - file missing, empty or refused)'}",
                  file=sys.stderr)
        if c.map_record:
            self._map_rec = open(c.map_record, "w")
            self._map_rec.write(self.map_header())
        if c.map_replay:
            self._map_rep = open(c.map_replay)
            head = [self._map_rep.readline() for _ in range(self.n_layers + 1)]
            if "".join(head) != self.map_header():
                raise MoeError(-6, f"map replay {c.map_replay}: the header does not match this stack")
        if c.route_trace:
            self._trace = open(c.route_trace, "w")
        self._map_frame()

    def _map_frame(self):
        """After every step (and once at start): replay -- read the frame of
        this step and place it (uploads of the experts a slot does not hold
        yet, then the tables); record -- write the published placement
        (patches/0008:440-489)."""
        if self._map_rep is not None:
            steps = self.stats()["steps"]
            head = self._map_rep.readline().split()
            if head != ["step", str(steps)]:
                raise MoeError(-6, f"map replay: expected frame 'step {steps}', read {' '.join(head)!r}")
            torch.cuda.synchronize(self.device)   # no upload may land after the placement
            for il in range(self.n_layers):
                toks = self._map_rep.readline().split()
                if len(toks) != 2 + self.ns[il] or toks[:2] != ["map", str(il)]:
                    raise MoeError(-6, f"map replay: bad frame line for layer {il}")
                self.place(il, [int(v) for v in toks[2:]], copy=True)
        if self._map_rec is not None:
            self._map_rec.write(self.map_frame())
            self._map_rec.flush()

    def _trace_routes(self, layer_ids, slots):
        """Route trace lines "route <steps> <layer> <n_ids> <n_tokens> id:slot
        ..." (patches/0008:508-518): layer_ids {layer: ids [n_tok, n_used]},
        slots {layer: expert -> slot (-1 absent)} as the router saw them."""
        steps = self.stats()["steps"]
        for il, ids in layer_ids.items():
            ids = np.asarray(ids).reshape(-1, self.n_used)
            es = slots[il]
            body = " ".join(f"{int(e)}:{int(es[e])}" for e in ids.ravel())
            self._trace.write(f"route {steps} {il} {self.n_used} {ids.shape[0]} {body}\n")

    def close(self):
        for f in (self._map_rec, self._map_rep, self._trace):
            if f is not None:
                f.close()
        self._map_rec = self._map_rep = self._trace = None
        if getattr(self, "ctx", None):
            self.lib.moe_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ck(self, rc, what):
        return check(rc, self.ctx, what)

    # -- weights --------------------------------------------------------------
    def layer_info(self, layer):
        info = MoeLayerInfo()
        self._ck(self.lib.moe_get_layer(self.ctx, layer, C.byref(info)), "moe_get_layer")
        return info

    def slot_views(self, layer):
        """torch uint8 views of the layer's gate/up/down slot slabs
        [n_slots + 1, bytes]."""
        info = self.layer_info(layer)
        n = info.n_slots + 1
        g = torch.as_tensor(_CudaView(info.gate_c, n * self.gate_bytes), device=self.device)
        u = torch.as_tensor(_CudaView(info.up_c, n * self.gate_bytes), device=self.device)
        d = torch.as_tensor(_CudaView(info.down_c, n * self.down_bytes), device=self.device)
        return g.view(n, -1), u.view(n, -1), d.view(n, -1)

    def set_router(self, layer, w):
        w = w.contiguous().float()
        self._ck(self.lib.moe_set_router(self.ctx, layer, _ptr(w)), "moe_set_router")

    def set_expert_weights(self, layer, gate, up, down):
        """Host copies of all experts of a layer (uint8, ggml layout), kept
        alive by this object; registered (pinned, mapped) by the library."""
        self._host[layer] = (gate, up, down)
        self._ck(self.lib.moe_set_expert_weights(self.ctx, layer, _ptr(gate), _ptr(up), _ptr(down)),
                 "moe_set_expert_weights")

    def set_shared_expert(self, layer, gate, up, down):
        """The always-on shared expert of a layer (n_shared == 1): uint8 gate,
        up, down bytes in ggml layout, host or device; copied by the library."""
        self._ck(self.lib.moe_set_shared_expert(self.ctx, layer, _ptr(gate), _ptr(up), _ptr(down)),
                 "moe_set_shared_expert")

    def place(self, layer, slot_expert, copy=True):
        se = np.ascontiguousarray(slot_expert, np.int32)
        self._ck(self.lib.moe_place(self.ctx, layer, _ptr(se), int(copy)), "moe_place")

    def synth_resident(self, seed=0, sigma=0.02, router_sigma=0.02, keep_router=False):
        """Every layer: synthetic N(0, sigma^2) experts generated on the device
        straight into slots 0..n_expert-1 (needs n_slots >= n_expert) and an
        fp32 N(0, router_sigma^2) router; experts placed identity.  With
        keep_router the router tensors stay in self.routers.  With a shared
        expert, its gate/up/down come from seeds base + 4, 5, 6 (self.shared
        keeps them when keep_router)."""
        self.routers = [] if keep_router else None
        self.shared = [] if keep_router and self.n_shared else None
        for il in range(self.n_layers):
            if self.ns[il] < self.n_expert:
                raise ValueError("synth_resident needs n_slots >= n_expert")
            info = self.layer_info(il)
            nbg = self.n_expert * self.gate_bytes // Q4K_BYTES
            nbd = self.n_expert * self.down_bytes // (Q6K_BYTES if self.down_type == QTYPE_Q6_K
                                                      else Q4K_BYTES)
            s = _stream()
            base = (seed + 1000 * il) & 0xFFFFFFFF
            self._ck(self.lib.moe_synth_weights(info.gate_c, nbg, QTYPE_Q4_K, base + 0, sigma, s), "synth")
            self._ck(self.lib.moe_synth_weights(info.up_c, nbg, QTYPE_Q4_K, base + 1, sigma, s), "synth")
            self._ck(self.lib.moe_synth_weights(info.down_c, nbd, self.down_type, base + 2, sigma, s),
                     "synth")
            r = torch.empty(self.n_expert, self.n_embd, device=self.device)
            self._ck(self.lib.moe_synth_f32(_ptr(r), r.numel(), base + 3, router_sigma, s), "synth")
            torch.cuda.synchronize(self.device)
            self.set_router(il, r)
            if keep_router:
                self.routers.append(r)
            se = list(range(self.n_expert)) + [-1] * (self.ns[il] - self.n_expert)
            self.place(il, se, copy=False)
            if self.n_shared:
                parts = []
                for off, nbytes, qt in ((4, self.gate_bytes, QTYPE_Q4_K), (5, self.gate_bytes, QTYPE_Q4_K),
                                        (6, self.down_bytes, self.down_type)):
                    t = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                    bb = Q4K_BYTES if qt == QTYPE_Q4_K else Q6K_BYTES
                    self._ck(self.lib.moe_synth_weights(_ptr(t), nbytes // bb, qt, base + off, sigma, s),
                             "synth")
                    parts.append(t)
                torch.cuda.synchronize(self.device)
                self.set_shared_expert(il, *parts)
                if self.shared is not None:
                    self.shared.append(tuple(parts))

    # -- hot path -------------------------------------------------------------
    def layer_forward(self, layer, x, stream=None):
        """x [n_tok, n_embd] fp32 (device) -> (y, ids, w)."""
        self.start()
        slots = {layer: self.tables(layer)["expert_slot"]} if self._trace is not None else None
        x = x.contiguous()
        n_tok = x.shape[0]
        y = torch.empty_like(x)
        ids = torch.empty(n_tok, self.n_used, dtype=torch.int32, device=x.device)
        w = torch.empty(n_tok, self.n_used, dtype=torch.float32, device=x.device)
        self._ck(self.lib.moe_layer_forward(self.ctx, layer, _ptr(x), _ptr(y), n_tok, _ptr(ids),
                                            _ptr(w), _stream(stream)), "moe_layer_forward")
        if slots is not None:
            self._trace_routes({layer: ids.cpu().numpy()}, slots)
        return y, ids, w

    def layer_forward_path(self, layer, x, path="auto", stream=None):
        """layer_forward with the expert arithmetic chosen: "gemv" (Q8_1
        activations, int8 dots), "gemm" (tcgen05 grouped GEMM, fp16 operands,
        fp32 sums) or "auto" (GEMM when the batch gives >= 4 pairs per expert)."""
        x = x.contiguous()
        n_tok = x.shape[0]
        y = torch.empty_like(x)
        ids = torch.empty(n_tok, self.n_used, dtype=torch.int32, device=x.device)
        w = torch.empty(n_tok, self.n_used, dtype=torch.float32, device=x.device)
        code = {"auto": 0, "gemv": 1, "gemm": 2}[path]
        self._ck(self.lib.moe_layer_forward_path(self.ctx, layer, _ptr(x), _ptr(y), n_tok, _ptr(ids),
                                                 _ptr(w), code, _stream(stream)), "moe_layer_forward_path")
        return y, ids, w

    def layer_forward_noalloc(self, layer, x, y, ids=None, w=None, stream=None):
        """layer_forward for callers that cannot allocate device memory while
        they run (their device memory is committed up front).  Neither the
        library nor this method allocates.  The caller owns y
        [n_tok, n_embd], and ids/w [n_tok, n_used] when it wants them.  The
        scratch is one static array per device, shared by every stack on that
        device: calls that overlap in time race on it.  n_tok is limited by
        its size (MOE_NOALLOC_SCRATCH_BYTES); a larger batch raises
        MoeError.  Returns y."""
        for t in (x, y, ids, w):
            if t is not None and not t.is_contiguous():
                raise ValueError("layer_forward_noalloc needs contiguous tensors (a copy would allocate)")
        self._ck(self.lib.moe_layer_forward_noalloc(self.ctx, layer, _ptr(x), _ptr(y), x.shape[0],
                                                    _ptr(ids), _ptr(w), _stream(stream)),
                 "moe_layer_forward_noalloc")
        return y

    def decode(self, h, out=None, debug=False, stream=None, profile=False, starve=0, spec=0):
        """Batch-1 decode of h [n_tok, n_embd] (device) through every layer,
        one token after another; returns out (and the per-layer dumps when
        debug; with profile, dumps["prof"] holds the per-CTA phase timestamps
        [n_tok, n_layers, 12, grid] in ns).  starve = r + 1 is for tests of
        the watchdog: rank r's first activation wait can then only run out.
        spec: the early gate/up copies, 0 on (default), 1 off, 2 on with a
        wrong prediction in every other (token, layer) (tests of the
        re-issue); the results are the same bits in every mode."""
        self.start()
        h = h.contiguous()
        n_tok = h.shape[0]
        out = torch.empty_like(h) if out is None else out
        dbg = None
        dumps = None
        trace = self._trace is not None
        if trace:   # the routed ids are needed: take the dumps, return them only on request
            slots = {il: self.tables(il)["expert_slot"] for il in range(self.n_layers)}
            want_dumps, debug = debug, True
        if debug:
            L, K, H = self.n_layers, self.n_used, self.n_embd
            dumps = {
                "x": torch.empty(n_tok, L, H, device=h.device),
                "ids": torch.empty(n_tok, L, K, dtype=torch.int32, device=h.device),
                "w": torch.empty(n_tok, L, K, device=h.device),
                "y": torch.empty(n_tok, L, H, device=h.device),
            }
            prof_ptr = None
            if profile:
                grid = self.decode_info()["grid"]
                dumps["prof"] = torch.zeros(n_tok, L, 12, grid, dtype=torch.int64, device=h.device)
                prof_ptr = dumps["prof"].data_ptr()
            dbg = MoeDecodeDbg(dumps["x"].data_ptr(), dumps["ids"].data_ptr(),
                               dumps["w"].data_ptr(), dumps["y"].data_ptr(), prof_ptr, starve, spec)
        elif starve or spec:
            dbg = MoeDecodeDbg(None, None, None, None, None, starve, spec)
        self._ck(self.lib.moe_decode(self.ctx, _ptr(h), _ptr(out), n_tok,
                                     C.byref(dbg) if dbg is not None else None, _stream(stream)),
                 "moe_decode")
        if trace:
            ids = dumps["ids"].cpu().numpy()   # [n_tok, L, k]
            self._trace_routes({il: ids[:, il] for il in range(self.n_layers)}, slots)
            debug = want_dumps
        return (out, dumps) if debug else out

    def decode_host(self, h_host, out_host, stream=None):
        """End to end: pinned host h -> device -> decode -> host out."""
        n_tok = h_host.shape[0]
        self._ck(self.lib.moe_decode_host(self.ctx, _ptr(h_host), _ptr(out_host), n_tok,
                                          _stream(stream)), "moe_decode_host")
        return out_host

    def sync(self, stream=None):
        self._ck(self.lib.moe_sync(self.ctx, _stream(stream)), "moe_sync")

    def set_wait_limit(self, ns):
        """Limit of the decode kernel's device waits in ns (0: the 2 s default)."""
        self._ck(self.lib.moe_set_wait_limit(self.ctx, int(ns)), "moe_set_wait_limit")

    def decode_info(self):
        out = np.zeros(5, np.int32)
        self._ck(self.lib.moe_decode_info(self.ctx, _ptr(out), 5), "moe_decode_info")
        return dict(zip(["grid", "smem_bytes", "gu_rows_max", "dn_rows_max", "threads"],
                        (int(v) for v in out)))

    # -- slot cache -----------------------------------------------------------
    def observe(self, layer, ids, stream=None):
        ids = ids.contiguous().to(torch.int32)
        ids2 = ids.view(1, -1) if ids.dim() == 1 else ids
        self._ck(self.lib.moe_observe(self.ctx, layer, _ptr(ids2), ids2.shape[0], ids2.shape[1],
                                      _stream(stream)), "moe_observe")

    def set_evictor(self, model):
        """LLAMA_MOE_EVICTOR: `model` (a predictor.MoePredictor, MOEP v3)
        scores each layer's resident experts at every step, and the victim is
        the lowest score instead of the least recently used slot.  None
        removes it."""
        if model is None:
            self._ck(self.lib.moe_set_evictor(self.ctx, 0, None, 0, None, None, None, None), "moe_set_evictor")
            return
        from .predictor import BLOCK_BELOW, BLOCK_CUR, BLOCK_PREV, BLOCK_SELF_PREV
        lo = np.ascontiguousarray(model.layer_of, np.int32)
        off = np.array([model.off[BLOCK_PREV], model.off[BLOCK_CUR], model.off[BLOCK_BELOW],
                        model.off[BLOCK_SELF_PREV]], np.int32)
        w = np.ascontiguousarray(model.w, np.float32)
        b = np.ascontiguousarray(model.bias, np.float32)
        pr = np.ascontiguousarray(model.prior, np.float32)
        self._ck(self.lib.moe_set_evictor(self.ctx, len(lo), _ptr(lo), int(model.feat_dim), _ptr(off),
                                          _ptr(w), _ptr(b), _ptr(pr)), "moe_set_evictor")

    def set_predictor(self, fn):
        """The predictor hook (cpp/moe-predictor.h as moe_obs_cb calls it):
        fn(layer, cur, next_prev, k) -> up to k expert ids for layer + 1,
        called after each single-token layer of layer_forward / observe.
        With early issue they become speculative uploads.  None removes it."""
        if fn is None:
            self._pred_cb = None
            self._ck(self.lib.moe_set_predictor(self.ctx, None, None), "moe_set_predictor")
            return

        def cb(ud, layer, cur, n_cur, nprev, n_nprev, out, k):
            try:
                got = list(fn(layer, [cur[i] for i in range(n_cur)], [nprev[i] for i in range(n_nprev)], k))[:k]
            except Exception as e:   # a raising hook predicts nothing
                print(f"moe predictor hook raised {e!r}", file=sys.stderr)
                return 0
            for i, v in enumerate(got):
                out[i] = int(v)
            return len(got)
        self._pred_cb = _lib.PREDICT_FN(cb)
        self._ck(self.lib.moe_set_predictor(self.ctx, C.cast(self._pred_cb, C.c_void_p), None),
                 "moe_set_predictor")

    def set_observe_hook(self, fn):
        """fn(layer, ids [n_tok, n_ids] numpy) after each observed layer
        (ggml_set_moe_obs_callback's callback).  None removes it."""
        if fn is None:
            self._obs_cb = None
            self._ck(self.lib.moe_set_observe_hook(self.ctx, None, None), "moe_set_observe_hook")
            return

        def cb(ud, layer, ids, n_tok, n_ids):
            try:
                fn(layer, np.ctypeslib.as_array(ids, shape=(n_tok * n_ids,)).copy().reshape(n_tok, n_ids))
            except Exception as e:
                print(f"moe observe hook raised {e!r}", file=sys.stderr)
        self._obs_cb = _lib.OBSERVE_FN(cb)
        self._ck(self.lib.moe_set_observe_hook(self.ctx, C.cast(self._obs_cb, C.c_void_p), None),
                 "moe_set_observe_hook")

    def step(self, stream=None):
        """llama_moe_cache_step: publish, schedule, flush (moe_step); then, as
        the reference, the heat file every 512 steps (patches/0007:749-753)
        and the map frame of this step."""
        self.start()
        self._ck(self.lib.moe_step(self.ctx, _stream(stream)), "moe_step")
        c = self.cache
        if c.heat_file and not c.freeze and self.stats()["steps"] % 512 == 0:
            try:
                save_heat(c.heat_file, np.stack([self.gate_state(il)["use_count"]
                                                 for il in range(self.n_layers)]))
            except OSError:
                print(f"moe-cache: heat file write FAILED: {c.heat_file}", file=sys.stderr)
        self._map_frame()
        if self._trace is not None:
            self._trace.flush()

    def tables(self, layer):
        ns = self.ns[layer]
        es = np.empty(self.n_expert, np.int32)
        se = np.empty(ns, np.int32)
        lu = np.empty(ns, np.uint64)
        fl = np.empty(ns, np.uint8)
        pr = np.empty(ns, np.uint64)
        self._ck(self.lib.moe_get_tables(self.ctx, layer, _ptr(es), _ptr(se), _ptr(lu), _ptr(fl),
                                         _ptr(pr)), "moe_get_tables")
        return {"expert_slot": es, "slot_expert": se, "last_use": lu, "in_flight": fl,
                "protect": pr}

    def gate_state(self, layer):
        E = self.n_expert
        heat = np.zeros(E, np.float32)
        ml = np.zeros(E, np.uint64)
        mp = np.zeros(E, np.uint64)
        uc = np.zeros(E, np.uint32)
        self._ck(self.lib.moe_get_gate_state(self.ctx, layer, _ptr(heat), _ptr(ml), _ptr(mp),
                                             _ptr(uc)), "moe_get_gate_state")
        return {"heat": heat, "miss_last": ml, "miss_prev": mp, "use_count": uc}

    def stats(self):
        out = np.zeros(len(STAT_NAMES), np.uint64)
        self._ck(self.lib.moe_get_stats(self.ctx, _ptr(out), len(STAT_NAMES)), "moe_get_stats")
        return {k: int(v) for k, v in zip(STAT_NAMES, out)}

    def stream_stats(self):
        """Just-in-time streaming counters (moe_stream_stats), by name."""
        out = np.zeros(len(STREAM_STAT_NAMES), np.uint64)
        self._ck(self.lib.moe_stream_stats(self.ctx, _ptr(out), len(STREAM_STAT_NAMES)), "moe_stream_stats")
        return {k: int(v) for k, v in zip(STREAM_STAT_NAMES, out)}

    def warm_start(self, use_count):
        uc = np.ascontiguousarray(use_count, np.uint32)
        return self._ck(self.lib.moe_warm_start(self.ctx, _ptr(uc)), "moe_warm_start")

    # -- diagnostics in the reference's text formats ----------------------------
    def map_header(self):
        """"moe-map 1" header (patches/0008:417-433)."""
        lines = [f"moe-map 1 {self.n_layers}"]
        lines += [f"layer {il} {self.ns[il]} {self.n_expert}" for il in range(self.n_layers)]
        return "\n".join(lines) + "\n"

    def map_frame(self, n_steps=None):
        """One "step / map" frame of the published placement (patches/0008:476-488)."""
        if n_steps is None:
            n_steps = self.stats()["steps"]
        lines = [f"step {n_steps}"]
        for il in range(self.n_layers):
            es = self.tables(il)["expert_slot"]
            pub = [-1] * self.ns[il]
            for e, s in enumerate(es):
                if s >= 0:
                    pub[s] = e
            lines.append("map %d" % il + "".join(f" {e}" for e in pub))
        return "\n".join(lines) + "\n"


def load_heat(path, n_layers, n_expert):
    """Parse a "moe-heat 1 <layers> <experts>" file (patches/0007:431-466):
    counts halved on load; refused (None) when the dimensions differ."""
    try:
        with open(path) as f:
            toks = f.read().split()
    except OSError:
        return None
    if len(toks) < 4 or toks[0] != "moe-heat":
        return None
    try:
        ver, nl, ne = int(toks[1]), int(toks[2]), int(toks[3])
    except ValueError:
        return None
    if ver != 1 or nl != n_layers or ne != n_expert:
        return None
    out = np.zeros((n_layers, n_expert), np.uint32)
    rest = toks[4:]
    for i in range(0, len(rest) - 2, 3):
        try:
            il, e, c = int(rest[i]), int(rest[i + 1]), int(rest[i + 2])
        except ValueError:
            break
        if 0 <= il < n_layers and 0 <= e < n_expert:
            out[il, e] = c // 2
    return out


def save_heat(path, counts):
    """Write counts [layers, experts] as "moe-heat 1" via temp + rename
    (patches/0007:468-485)."""
    import os
    counts = np.asarray(counts)
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        f.write(f"moe-heat 1 {counts.shape[0]} {counts.shape[1]}\n")
        for il in range(counts.shape[0]):
            for e in range(counts.shape[1]):
                if counts[il, e]:
                    f.write(f"{il} {e} {int(counts[il, e])}\n")
    os.replace(tmp, path)
