"""Generate the golden fixtures in tests/golden/ (run here, where the
reference tree and gguf-py are available; the fixtures travel, the sources
do not).

  q4k_q6k_gguf.npz     blocks produced by our quantiser and their decode by
                       gguf-py 0.19.0 (gguf.quants.Q4_K / Q6_K
                       .dequantize_blocks) -- the third-party decoder of the
                       ggml block formats, named and version-pinned.
  greedy_alloc.json    inputs and outputs of the reference's own
                       greedy_allocate_bytes (experiments/p7_slot_allocation.py
                       :144-185), imported from the reference tree.
  predictor_toy.bin    a small MOEP v3 file written by our writer, and
  predictor_toy.json   the scores / top-k / update results of the reference's
                       own cpp/moe-predictor.cpp (compiled into oracle/_ref by
                       oracle/Makefile) on it.
  expert_cache.json    a scripted prefetch / admit / query sequence through the
                       reference's own ExpertCache (src/prefetch_engine.py),
                       its CUDA stream calls replaced by host stand-ins.

    python tests/golden/make_golden.py [gguf greedy predictor expert_cache]
"""
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.oracle import reference_dir  # noqa: E402

REF = reference_dir()


def gguf_fixture():
    import gguf
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    import oracle
    rng = np.random.default_rng(2024)
    out = {"gguf_version": getattr(gguf, "__version__", "0.19.0")}
    for name, qt, gt in (("q4k", 12, T.Q4_K), ("q6k", 14, T.Q6_K)):
        x = (rng.standard_normal(256 * 16) * 0.02).astype(np.float32)
        x[:256] = 0.0
        blocks = oracle.quantize(x, qt)
        out[f"{name}_x"] = x
        out[f"{name}_blocks"] = blocks
        out[f"{name}_deq"] = quants.dequantize(blocks, gt).ravel().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_q6k_gguf.npz"), **out)


def greedy_fixture():
    path = os.path.join(REF, "experiments", "p7_slot_allocation.py")
    spec = importlib.util.spec_from_file_location("p7_ref", path)
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, os.path.join(REF, "experiments"))
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(7)
    cases = []
    for case in range(6):
        n_layers = [8, 16, 48, 48, 12, 5][case]
        grid = [[16, 32, 56, 96], [8, 16, 24, 32, 48, 64], [16, 32, 56, 96],
                [24, 40, 56, 72, 96, 128], [16, 56], [4, 8, 16]][case]
        uniform = [32, 16, 56, 56, 16, 8][case]
        frozen = [[], [3], [47], [0, 47], [], [2]][case]
        miss = {}
        base = rng.uniform(0.2, 1.5, n_layers)
        for i, g in enumerate(grid):
            miss[g] = [float(b * np.exp(-g / rng.uniform(20, 60))) for b in base]
        if case == 4:
            miss[grid[1]][1] = miss[grid[0]][1]        # a flat step (zero value)
        eb = [float(b) for b in rng.choice([2654208.0, 3059712.0], n_layers)]
        if case == 3:
            eb[5] = 0.0                                  # unknown size -> mean
        cap, used, budget = mod.greedy_allocate_bytes(miss, grid, n_layers, uniform, frozen, eb)
        cases.append({"miss8": {str(k): v for k, v in miss.items()}, "grid": grid,
                      "n_layers": n_layers, "uniform_cap": uniform, "frozen": frozen,
                      "expert_bytes": eb, "cap": cap, "used": used, "budget": budget})
    with open(os.path.join(HERE, "greedy_alloc.json"), "w") as f:
        json.dump({"source": "experiments/p7_slot_allocation.py:144-185 (reference)",
                   "cases": cases}, f)


def predictor_fixture():
    import oracle
    from moe_prefetch_b200.predictor import (BLOCK_BELOW, BLOCK_CUR, BLOCK_PREV,
                                             BLOCK_SELF_PREV, MoePredictor)
    oracle.build()
    rng = np.random.default_rng(11)
    E, n_layers = 32, 5
    p = MoePredictor()
    p.n_expert, p.n_layers, p.top_k, p.feat_dim = E, n_layers, 8, 4 * E
    p.off = {0: -1, BLOCK_PREV: 0, BLOCK_CUR: E, BLOCK_BELOW: 2 * E, BLOCK_SELF_PREV: 3 * E}
    p.layer_of = np.array([0, 1, 3], np.int32)
    p.prior = np.array([0.0, 0.5, 1.25], np.float32)
    p.bias = rng.standard_normal((3, E)).astype(np.float32)
    p.w = (rng.standard_normal((3, 4 * E, E)) * 0.3).astype(np.float32)
    path = os.path.join(HERE, "predictor_toy.bin")
    p.save(path)
    ref = oracle.RefPredictor(path)
    cases = []
    for il in (0, 1, 3):
        for _ in range(4):
            ins = {k: [int(v) for v in rng.choice(E, rng.integers(0, 9), replace=True)]
                   for k in ("prev", "cur", "below", "self_prev")}
            s = ref.score(il, **ins)
            top = ref.top_k_ids(s, 8)
            cases.append({"layer": il, "inputs": ins, "scores": s.tolist(), "top8": top.tolist()})
    # one online update, then scores again
    truth = [1, 5, 9, 13, 17, 21, 25, 29]
    ins = {"prev": [2, 4], "cur": [1, 3, 5], "below": [], "self_prev": [7]}
    hit = ref.update(1, truth, 0.05, **ins)
    after = ref.score(1, **ins)
    with open(os.path.join(HERE, "predictor_toy.json"), "w") as f:
        json.dump({"source": "cpp/moe-predictor.cpp (reference, via oracle/_ref)",
                   "cases": cases,
                   "update": {"layer": 1, "truth": truth, "lr": 0.05, "inputs": ins,
                              "hit": hit, "scores_after": after.tolist()}}, f)


class _CpuStream:
    """Stand-in for torch.cuda.Stream on a host without a GPU: copies are
    synchronous, so every recorded event has completed."""

    def __init__(self, device=None):
        pass

    def synchronize(self):
        pass


class _DoneEvent:
    def record(self, stream=None):
        pass

    def query(self):
        return True


def _cpu_torch():
    """The real torch module with its CUDA stream / event / pinned-memory
    calls replaced by host stand-ins, so that the reference's ExpertCache runs
    its own bookkeeping unchanged on the CPU."""
    import contextlib
    import types

    import torch
    shim = types.ModuleType("torch")
    shim.__dict__.update({k: getattr(torch, k) for k in dir(torch) if not k.startswith("__")})

    def empty(*shape, device=None, pin_memory=False, **kw):
        return torch.empty(*shape, **kw)
    shim.empty = empty
    shim.cuda = types.SimpleNamespace(Stream=_CpuStream, Event=_DoneEvent,
                                      stream=lambda s: contextlib.nullcontext())
    return shim


def expert_cache_fixture():
    with open(os.path.join(HERE, "expert_cache.json"), "w") as f:
        json.dump(expert_cache_cases(), f)


def expert_cache_cases():
    """A scripted sequence of prefetch / admit / sync / query calls run
    through the reference's own ExpertCache (src/prefetch_engine.py:47-168),
    imported from the reference tree with host stand-ins for its CUDA calls.
    Recorded after every call: the return value, each layer's expert -> slot
    map in LRU order, and the statistics; at the end, which staging row every
    slot holds.  Queries follow a sync(), so no copy is in flight (no `late`:
    on a GPU that outcome depends on timing)."""
    path = os.path.join(REF, "src", "prefetch_engine.py")
    spec = importlib.util.spec_from_file_location("ref_prefetch_engine", path)
    mod = importlib.util.module_from_spec(spec)
    import torch
    shim = _cpu_torch()
    saved = sys.modules["torch"]
    sys.modules["torch"] = shim
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.modules["torch"] = saved
    cases = []
    for case, (L, E, cap, nb, steps) in enumerate(((3, 16, 5, 256, 120), (2, 128, 24, 4096, 200),
                                                    (1, 8, 8, 64, 60))):
        rng = np.random.default_rng(100 + case)
        xc = mod.ExpertCache(L, E, cap, device="cpu", bytes_per_expert=nb)
        # staging row e: bytes (e * 37 + j) % 251, so a slot's bytes name its expert
        xc.staging.copy_(torch.from_numpy(
            ((np.arange(E)[:, None] * 37 + np.arange(nb)[None, :]) % 251).astype(np.uint8)))
        ops = []
        for _ in range(steps):
            layer = int(rng.integers(L))
            kind = ("prefetch", "admit", "query")[int(rng.integers(3))]
            n = int(rng.integers(1, min(E, 12) + 1))
            ids = [int(v) for v in rng.integers(0, E, n)]   # duplicates included
            if kind == "prefetch":
                ret = xc.prefetch(layer, ids)
            elif kind == "admit":
                ret = xc.admit(layer, ids)
            else:
                xc.sync()
                ret = [list(v) for v in xc.query(layer, ids)]
            ops.append({"op": kind, "layer": layer, "ids": ids, "ret": ret,
                        "maps": [[[int(e), int(s)] for e, s in m.items()] for m in xc.maps],
                        "stats": dict(xc.stats)})
        xc.sync()
        held = [[int(xc.slabs[l][s][0]) for s in range(cap)] for l in range(L)]
        cases.append({"n_layers": L, "n_experts": E, "capacity": cap, "bytes_per_expert": nb,
                      "ops": ops, "summary": xc.summary(), "vram_bytes": xc.vram_bytes(),
                      "slab_first_byte": held})
    return {"source": "src/prefetch_engine.py:47-168 (reference ExpertCache, run on the host)",
            "cases": cases}


if __name__ == "__main__":
    which = sys.argv[1:] or ["gguf", "greedy", "predictor", "expert_cache"]
    if "gguf" in which:
        gguf_fixture()
    if "greedy" in which:
        greedy_fixture()
    if "predictor" in which:
        predictor_fixture()
    if "expert_cache" in which:
        expert_cache_fixture()
    print("golden fixtures written to", HERE)
