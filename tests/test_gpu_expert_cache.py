"""ExpertCache (moe_xc_* in the C ABI) against the reference's own
ExpertCache (src/prefetch_engine.py:47-168).

tests/golden/expert_cache.json holds a scripted sequence of prefetch / admit
/ sync / query calls run through the reference's class (on the host, its CUDA
stream calls replaced by stand-ins; tests/golden/make_golden.py).  Replayed
here on the GPU, every call must give the same return value, the same
expert -> slot map and the same statistics, and at the end every mapped slot
must hold its expert's staging bytes.  Queries follow a sync(), as in the
fixture, so that no copy is in flight and `late` cannot depend on timing.
"""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "expert_cache.json")


def _cases():
    with open(GOLD) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", range(3))
def test_expert_cache_matches_reference(case):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200.prefetch_engine import ExpertCache
    g = _cases()[case]
    L, E, cap, nb = g["n_layers"], g["n_experts"], g["capacity"], g["bytes_per_expert"]
    host = ((np.arange(E)[:, None] * 37 + np.arange(nb)[None, :]) % 251).astype(np.uint8)
    staging = torch.from_numpy(host).pin_memory()
    xc = ExpertCache(L, E, cap, bytes_per_expert=nb, staging=staging)
    try:
        for i, op in enumerate(g["ops"]):
            layer, ids = op["layer"], op["ids"]
            if op["op"] == "prefetch":
                assert xc.prefetch(layer, ids) == op["ret"], f"op {i}: prefetch count"
            elif op["op"] == "admit":
                xc.admit(layer, ids)
            else:
                xc.sync()
                hit, late, miss = xc.query(layer, ids)
                assert [hit, late, miss] == op["ret"], f"op {i}: query"
            for ll in range(L):
                want = {e: s for e, s in op["maps"][ll]}
                got = {e: xc.slot_of(ll, e) for e in range(E) if xc.slot_of(ll, e) >= 0}
                assert got == want, f"op {i}: layer {ll} expert -> slot map"
            assert xc.stats == op["stats"], f"op {i}: stats"
        xc.sync()
        assert xc.vram_bytes() == g["vram_bytes"]
        s = xc.summary()
        for k, v in g["summary"].items():
            assert s[k] == pytest.approx(v, rel=0, abs=0), k
        last = g["ops"][-1]["maps"]
        for ll in range(L):
            slab = xc.slabs[ll].cpu().numpy()
            for e, sl in last[ll]:
                assert int(slab[sl][0]) == g["slab_first_byte"][ll][sl]
                assert np.array_equal(slab[sl], host[e]), f"layer {ll} slot {sl} bytes"
    finally:
        xc.close()
