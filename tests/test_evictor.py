"""LLAMA_MOE_EVICTOR on the host side: the oracle's C restatement of
moe_predictor::score (cpp/moe-predictor.cpp:165-223) against our Python
scorer, the reference's golden fixture and, when oracle/_ref is built, the
reference's own compiled scorer on its shipped evictor; and the oracle's
victim choice (patches/0006:790-913, 0007:680-727): the lowest score, recency
breaking ties, empty / in-flight / protected slots as under LRU."""
import json
import os

import numpy as np
import pytest

from conftest import REFERENCE, toy_moep
from moe_prefetch_b200.predictor import MoePredictor

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def _inputs(rng, E, n=8):
    ins = {k: rng.choice(E, n, replace=False).astype(np.int32) for k in ("prev", "cur", "below", "self_prev")}
    ins["cur"][1] = ins["cur"][0]          # a repeated id adds its row twice
    ins["below"][2] = E + 3                # out of range: skipped
    ins["self_prev"][3] = -1
    return ins


@pytest.mark.parametrize("blocks,prior", [((1, 2, 3, 4), 0.25), ((2, 4), 0.0), ((4, 3, 2, 1), -0.5)])
def test_oracle_score_equals_python_bit_for_bit(oracle_lib, blocks, prior):
    E = 64
    m = toy_moep(4, E, [0, 2, 3], seed=len(blocks), blocks=blocks, prior=prior)
    rng = np.random.default_rng(1)
    for il in (0, 2, 3):
        for _ in range(5):
            ins = _inputs(rng, E)
            a = m.score(il, **ins)
            b = oracle_lib.evict_score(m, il, **ins)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), il
    ins = _inputs(rng, E)
    ins["prev"] = ins["prev"][:0]          # empty lists (the first token)
    assert np.array_equal(m.score(3, **ins).view(np.uint32), oracle_lib.evict_score(m, 3, **ins).view(np.uint32))


def test_oracle_score_matches_reference_golden(oracle_lib):
    p = MoePredictor.load(os.path.join(GOLD, "predictor_toy.bin"))
    with open(os.path.join(GOLD, "predictor_toy.json")) as f:
        g = json.load(f)
    for case in g["cases"]:
        s = oracle_lib.evict_score(p, case["layer"], **case["inputs"])
        np.testing.assert_allclose(s, np.array(case["scores"], np.float32), rtol=0, atol=2e-6)


def test_oracle_score_live_reference_evictor(oracle_lib):
    path = os.path.join(REFERENCE, "models", "evictor-real.bin")
    if not (os.path.exists(path) and oracle_lib.RefPredictor.available()):
        pytest.skip("reference models / oracle/_ref not present")
    ref = oracle_lib.RefPredictor(path)
    ours = MoePredictor.load(path)
    rng = np.random.default_rng(3)
    n = 0
    for il in range(ours.n_layers):
        if not ours.has_layer(il):
            continue
        ins = {k: rng.choice(ours.n_expert, 8, replace=False).astype(np.int32)
               for k in ("prev", "cur", "below", "self_prev")}
        a = oracle_lib.evict_score(ours, il, **ins)
        b = ref.score(il, **ins)
        # both built without fused multiply-adds, same sequential sums
        assert np.array_equal(a.view(np.uint32), np.asarray(b, np.float32).view(np.uint32)), il
        n += 1
    assert n > 0


def test_oracle_victim_is_lowest_score(oracle_lib):
    """One layer, 4 slots full, a miss to schedule: LRU would take the oldest
    slot, the evictor takes the resident expert with the lowest score."""
    E = 32
    m = toy_moep(1, E, [0], seed=5, blocks=(2,), prior=0.0)
    m.w[:] = 0.0                            # scores = the z-scored bias
    m.bias[0] = np.arange(E, dtype=np.float32)[::-1].copy()   # expert e scores E - 1 - e
    for use_model in (False, True):
        oc = oracle_lib.OracleCache(1, E, 4, max_inserts=1, admit_mode=0, batch_tables=True)
        if use_model:
            oc.set_evictor(m)
        for t, e in enumerate([3, 9, 20, 5]):   # fill: slot order 0..3, recency 3 < 9 < 20 < 5
            oc.observe(0, np.array([[e]], np.int32))
            oc.step()
        oc.observe(0, np.array([[7]], np.int32))   # a miss
        oc.step()                                  # scheduled
        oc.step()                                  # published
        se = oc.tables(0)["slot_expert"]
        assert 7 in se
        gone = ({3, 9, 20, 5} - set(se.tolist())).pop()
        assert gone == (20 if use_model else 3), (use_model, se)   # 20 has the lowest score
        oc.close()
