"""The predictor hook (MOEP v3): our reader/scorer pinned to the reference's
own cpp/moe-predictor.cpp -- through a golden fixture generated with it, and
live through oracle/_ref when the reference tree is present.  The format
checks follow the reference's tests/test_predictor_format.py."""
import json
import os

import numpy as np
import pytest

from moe_prefetch_b200.predictor import MoePredictor, MoepError

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
from conftest import REFERENCE  # noqa: E402

MODELS = os.path.join(REFERENCE, "models")


def test_scores_match_reference_golden():
    p = MoePredictor.load(os.path.join(GOLD, "predictor_toy.bin"))
    with open(os.path.join(GOLD, "predictor_toy.json")) as f:
        g = json.load(f)
    for case in g["cases"]:
        s = p.score(case["layer"], **case["inputs"])
        np.testing.assert_allclose(s, np.array(case["scores"], np.float32), rtol=0, atol=2e-6)
        assert list(p.top_k_ids(np.array(case["scores"], np.float32), 8)) == case["top8"]
    u = g["update"]
    hit = p.update(u["layer"], u["truth"], u["lr"], **u["inputs"])
    assert abs(hit - u["hit"]) < 1e-7
    np.testing.assert_allclose(p.score(u["layer"], **u["inputs"]),
                               np.array(u["scores_after"], np.float32), atol=2e-5)


def test_round_trip_is_exact(tmp_path):
    p = MoePredictor.load(os.path.join(GOLD, "predictor_toy.bin"))
    out = str(tmp_path / "m.bin")
    p.save(out)
    assert open(out, "rb").read() == open(os.path.join(GOLD, "predictor_toy.bin"), "rb").read()


def test_rejects_bad_files(tmp_path):
    src = open(os.path.join(GOLD, "predictor_toy.bin"), "rb").read()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(MoepError, match="not a MOEP"):
        MoePredictor.load(str(bad))
    bad.write_bytes(src[: len(src) // 2])
    with pytest.raises(MoepError, match="truncated"):
        MoePredictor.load(str(bad))
    bad.write_bytes(src + b"x")
    with pytest.raises(MoepError, match="trailing"):
        MoePredictor.load(str(bad))
    v2 = bytearray(src)
    v2[4] = 2
    bad.write_bytes(bytes(v2))
    with pytest.raises(MoepError, match="version"):
        MoePredictor.load(str(bad))


@pytest.mark.parametrize("name", ["predictor-real.bin", "predictor-fresh.bin", "evictor-real.bin"])
def test_live_reference_models(oracle_lib, name):
    path = os.path.join(MODELS, name)
    if not (os.path.exists(path) and oracle_lib.RefPredictor.available()):
        pytest.skip("reference models / oracle/_ref not present")
    ref = oracle_lib.RefPredictor(path)
    ours = MoePredictor.load(path)
    assert ours.n_expert == ref.n_expert and ours.feat_dim == ref.feat_dim
    rng = np.random.default_rng(0)
    for il in range(ours.n_layers):
        if not ours.has_layer(il):
            assert not ref.has_layer(il)
            continue
        ins = {k: rng.choice(ours.n_expert, 8, replace=False) for k in
               ("prev", "cur", "below", "self_prev")}
        a = ours.score(il, **ins)
        b = ref.score(il, **ins)
        np.testing.assert_allclose(a, b, atol=2e-4)        # cpp/verify_against_python.py:97
        assert list(ours.top_k_ids(a, 8)) == list(ref.top_k_ids(b, 8))
