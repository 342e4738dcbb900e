"""ExpertCache: the reference's PyTorch prototype API (src/prefetch_engine.py),
backed by the C ABI of libmoeb200.so.

Same constructor, methods and return shapes as the reference:
``prefetch(layer, ids) -> int``, ``query(layer, ids) -> (hit, late, miss)``,
``admit(layer, ids)``, ``sync()``, ``vram_bytes()``, ``summary()``.
Per layer a fixed ``[capacity, bytes_per_expert]`` slab in device memory and
an LRU expert -> slot map; copies run from a pinned host staging buffer on a
dedicated non-blocking stream, one event per copy, so a copy still in flight
at query time reports as ``late``, not as a hit (src/prefetch_engine.py:108-132).
"""
import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import check

EXPERT_MIB = 2.92                       # src/prefetch_engine.py:41
EXPERT_BYTES = int(EXPERT_MIB * 1024 * 1024)


class _View:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


class ExpertCache:
    """Per-layer LRU cache of experts resident in VRAM, with async refill."""

    def __init__(self, n_layers, n_experts, capacity, device="cuda",
                 bytes_per_expert=EXPERT_BYTES, staging=None):
        self.lib = _lib.load()
        self.n_layers = n_layers
        self.n_experts = n_experts
        self.capacity = capacity
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.bytes_per_expert = bytes_per_expert
        # host staging, pinned; content is the caller's (or zeros)
        if staging is None:
            staging = torch.zeros((n_experts, bytes_per_expert), dtype=torch.uint8,
                                  pin_memory=True)
        self.staging = staging
        h = C.c_void_p()
        check(self.lib.moe_xc_create(n_layers, n_experts, capacity, bytes_per_expert,
                                     C.c_void_p(staging.data_ptr()), self.device.index,
                                     C.byref(h)), None, "moe_xc_create")
        self.h = h
        self.slabs = [
            torch.as_tensor(_View(self.lib.moe_xc_slab(self.h, layer),
                                  capacity * bytes_per_expert),
                            device=self.device).view(capacity, bytes_per_expert)
            for layer in range(n_layers)]

    def close(self):
        if getattr(self, "h", None):
            self.slabs = []
            self.lib.moe_xc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _ids(expert_ids):
        a = np.ascontiguousarray([int(e) for e in expert_ids], np.int32)
        return a, a.ctypes.data_as(C.c_void_p)

    # -- public ------------------------------------------------------------
    def prefetch(self, layer, expert_ids):
        """Start async copies for `expert_ids` into layer's cache. Returns count."""
        a, p = self._ids(expert_ids)
        return check(self.lib.moe_xc_prefetch(self.h, layer, p, len(a)), None, "prefetch")

    def query(self, layer, expert_ids):
        """Which of `expert_ids` are usable NOW, without waiting?  A copy still
        in flight is `late`, not a hit."""
        a, p = self._ids(expert_ids)
        st = np.empty(len(a), np.int32)
        check(self.lib.moe_xc_query(self.h, layer, p, len(a), st.ctypes.data_as(C.c_void_p)),
              None, "query")
        hit = [int(e) for e, s in zip(a, st) if s == 0]
        late = [int(e) for e, s in zip(a, st) if s == 1]
        miss = [int(e) for e, s in zip(a, st) if s == 2]
        return hit, late, miss

    def admit(self, layer, expert_ids):
        """A miss was computed elsewhere; bring it in so the next token can use
        it.  This moves the bytes."""
        a, p = self._ids(expert_ids)
        check(self.lib.moe_xc_admit(self.h, layer, p, len(a)), None, "admit")

    def sync(self):
        check(self.lib.moe_xc_sync(self.h), None, "sync")

    def vram_bytes(self):
        return int(self.lib.moe_xc_vram_bytes(self.h))

    def slot_of(self, layer, expert):
        return int(self.lib.moe_xc_slot_of(self.h, layer, expert))

    @property
    def stats(self):
        out = np.zeros(6, np.uint64)
        check(self.lib.moe_xc_stats(self.h, out.ctypes.data_as(C.c_void_p)), None, "stats")
        return dict(zip(["hits", "misses", "late", "fetches", "bytes", "evictions"],
                        (int(v) for v in out)))

    def summary(self):
        s = dict(self.stats)
        total = s["hits"] + s["misses"] + s["late"]
        s["expert_hit_rate"] = s["hits"] / max(total, 1)
        s["late_rate"] = s["late"] / max(total, 1)
        s["gb_moved"] = s["bytes"] / 1e9
        return s
