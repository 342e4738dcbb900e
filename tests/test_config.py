"""Host configuration logic: the reference's CLI/env switches, slot profiles,
and the byte-priced greedy allocator pinned to the reference's own Python
function (golden fixture from experiments/p7_slot_allocation.py)."""
import json
import os

import pytest

from conftest import REFERENCE

from moe_prefetch_b200.config import (MoeCacheConfig, format_slot_profile,
                                      greedy_allocate_bytes, parse_slot_profile)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_env_defaults_match_reference():
    c = MoeCacheConfig.from_env({})
    # patches/0006:161 (max_inserts 2), 0007:188-193 (admit defaults)
    assert (c.max_inserts, c.admit_mode, c.admit_window, c.admit_half, c.admit_floor) == \
        (2, 0, 8, 64, 1.0)
    assert c.cache_prior == 0.0 and not c.batch_tables and not c.early_issue
    assert c.predict_top == 3


def test_env_parsing_rules(capsys):
    env = {"LLAMA_MOE_ADMIT": "window", "LLAMA_MOE_ADMIT_WINDOW": "0",
           "LLAMA_MOE_ADMIT_HALF": "-3", "LLAMA_MOE_CACHE_PRIOR": "-0.5",
           "LLAMA_MOE_BATCH_TABLES": "1", "LLAMA_MOE_SPEC_PROBATION": "7"}
    c = MoeCacheConfig.from_env(env, ["--moe-expert-cache", "56",
                                      "--moe-expert-cache-inserts", "3"])
    assert c.admit_mode == 2 and c.admit_window == 1 and c.admit_half == 1
    assert c.cache_prior == 0.0 and c.batch_tables and c.spec_probation
    assert c.n_slots == 56 and c.max_inserts == 3
    c = MoeCacheConfig.from_env({"LLAMA_MOE_ADMIT": "bogus"})
    assert c.admit_mode == 0
    assert "NOT UNDERSTOOD" in capsys.readouterr().err
    c = MoeCacheConfig.from_env({"LLAMA_MOE_ADMIT": "heat", "LLAMA_MOE_CACHE_FREEZE": "1"})
    assert c.admit_mode == 1 and c.max_inserts == 0
    c = MoeCacheConfig.from_env({"LLAMA_MOE_MAP_REPLAY": "/tmp/x"})
    assert c.freeze and c.max_inserts == 0
    c = MoeCacheConfig.from_env({}, ["--moe-expert-cache-inserts", "0"])
    assert c.max_inserts == 2          # non-positive keeps the default


def test_stream_env_rules():
    # patches/0010:969-975 defaults; 1828-1832 clamps; 1963 LLAMA_MOE_STREAM
    c = MoeCacheConfig.from_env({})
    assert not c.stream and (c.stream_per_layer, c.stream_reserve, c.stream_gbps, c.stream_topk) == \
        (4, 2, 45.7, 8)
    c = MoeCacheConfig.from_env({"LLAMA_MOE_STREAM": "1", "LLAMA_MOE_STREAM_TOPK": "12",
                                 "LLAMA_MOE_STREAM_PER_LAYER": "0", "LLAMA_MOE_STREAM_GBPS": "0.5",
                                 "LLAMA_MOE_STREAM_RESERVE": "-4"})
    assert c.stream and c.stream_topk == 8 and c.stream_per_layer == 1 and c.stream_gbps == 1.0
    assert c.stream_reserve == 0
    c = MoeCacheConfig.from_env({"LLAMA_MOE_STREAM": "0", "LLAMA_MOE_STREAM_TOPK": "-1"})
    assert not c.stream and c.stream_topk == 1


@pytest.mark.parametrize("spec,expect", [
    ("", {}),
    ("0:16,3:32", {0: 16, 3: 32}),
    ("0:16,3:32x,4:5", {0: 16, 3: 32}),      # stops at the malformed tail
    ("0:16,1:0,2:8", {0: 16}),               # n <= 0 stops parsing
    ("5: 12 ,6:7", {5: 12}),                 # %d skips leading blanks only
    (" 2:9", {2: 9}),
    ("abc", {}),
])
def test_slot_profile_parse(spec, expect):
    assert parse_slot_profile(spec) == expect


def test_slots_per_layer():
    c = MoeCacheConfig(n_slots=56, slot_profile="0:16,47:96")
    s = c.slots_per_layer(48, 128)
    assert s[0] == 16 and s[47] == 96 and s[1] == 56
    assert MoeCacheConfig().slots_per_layer(2, 128) == [128, 128]
    assert parse_slot_profile(format_slot_profile([3, 4, 5])) == {0: 3, 1: 4, 2: 5}


def _load_cases():
    with open(os.path.join(GOLD, "greedy_alloc.json")) as f:
        return json.load(f)["cases"]


def test_greedy_matches_reference_golden():
    for case in _load_cases():
        miss = {int(k): v for k, v in case["miss8"].items()}
        cap, used, budget = greedy_allocate_bytes(miss, case["grid"], case["n_layers"],
                                                  case["uniform_cap"], case["frozen"],
                                                  case["expert_bytes"])
        assert cap == case["cap"]
        assert used == case["used"] and budget == case["budget"]


def test_greedy_oracle_restatement_matches(oracle_lib):
    for case in _load_cases():
        miss = {int(k): v for k, v in case["miss8"].items()}
        cap, used, budget = oracle_lib.greedy_allocate_bytes(
            miss, case["grid"], case["n_layers"], case["uniform_cap"], case["frozen"],
            case["expert_bytes"])
        assert cap == case["cap"]
        assert abs(used - case["used"]) <= 1e-6 * case["used"]
        assert abs(budget - case["budget"]) <= 1e-6 * case["budget"]


def test_greedy_against_live_reference():
    path = os.path.join(REFERENCE, "experiments", "p7_slot_allocation.py")
    if not os.path.exists(path):
        pytest.skip("reference tree not present")
    import importlib.util
    import sys
    import numpy as np
    sys.path.insert(0, os.path.dirname(path))
    spec = importlib.util.spec_from_file_location("p7_live", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(99)
    for _ in range(20):
        n = int(rng.integers(3, 20))
        grid = sorted(set(int(v) for v in rng.integers(4, 128, int(rng.integers(2, 6)))))
        if len(grid) < 2:
            continue
        miss = {g: [float(v) for v in rng.uniform(0, 2, n) / (i + 1)] for i, g in enumerate(grid)}
        eb = [float(v) for v in rng.choice([0.0, 2.6e6, 3.06e6], n)]
        if not any(eb):
            eb[0] = 3.06e6
        frozen = [int(v) for v in rng.choice(n, int(rng.integers(0, 2)), replace=False)]
        uc = int(rng.choice(grid))
        assert greedy_allocate_bytes(miss, grid, n, uc, frozen, eb) == \
            tuple(mod.greedy_allocate_bytes(miss, grid, n, uc, frozen, eb))
