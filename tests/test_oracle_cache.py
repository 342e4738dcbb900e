"""The oracle's slot-table state machine pinned to scenarios read off the
reference patches: free-pool order, first empty slot then strict-LRU victim,
budget rules, second-miss window, heat gate, probation, freeze, deterministic
publication order, map/heat text formats, warm start."""
import os

import numpy as np

U64_MAX = np.uint64(0xFFFFFFFFFFFFFFFF)


def mk(oracle_lib, **kw):
    args = dict(n_layers=1, n_expert=8, n_slots=2, max_inserts=2, batch_tables=True)
    args.update(kw)
    return oracle_lib.OracleCache(**args)


def test_schedule_lru_and_publication(oracle_lib):
    """patches/0006:797-838 (victim: first empty non-in-flight slot, else
    strict-< LRU) and 0008:613-627 (publish in (layer, slot) order)."""
    c = mk(oracle_lib)
    c.observe(0, [3, 5, 6])
    c.step()                          # reversed pending: 6 -> slot 0, 5 -> slot 1
    j = c.jobs()
    assert [tuple(r[:3]) for r in j] == [(0, 6, 0), (0, 5, 1)]
    t = c.tables(0)
    assert list(t["in_flight"]) == [1, 1] and list(t["slot_expert"]) == [-1, -1]
    c.observe(0, [3, 5])              # 5 still in flight -> a miss again
    c.step()                          # publish (6,0) clock 1, (5,1) clock 2; then 5 resident
    t = c.tables(0)
    # pending reversed [5, 3]: 5 resident spends budget, 3 evicts LRU slot 0 (expert 6)
    assert list(t["slot_expert"]) == [-1, 5]
    assert list(t["last_use"]) == [1, 2]
    assert list(t["in_flight"]) == [1, 0]
    assert t["expert_slot"][6] == -1 and t["expert_slot"][5] == 1
    c.step()
    t = c.tables(0)
    assert list(t["slot_expert"]) == [3, 5] and list(t["last_use"]) == [3, 2]
    s = c.stats()
    assert (s["steps"], s["scheduled"], s["published"], s["clock"]) == (3, 3, 3, 3)
    assert (s["misses"], s["hits"]) == (5, 0)


def test_resident_pending_spends_budget(oracle_lib):
    """patches/0007:680-685: a pending id that became resident costs one insert."""
    c = mk(oracle_lib, n_expert=16, n_slots=4, max_inserts=1)
    c.observe(0, [7])
    c.step()                          # 7 -> slot 0
    c.observe(0, [9, 7])              # 7 in flight: miss; pending [9, 7]
    c.step()                          # publish 7; reversed: 7 resident -> budget 0
    assert c.jobs().shape[0] == 0
    assert c.tables(0)["expert_slot"][9] == -1


def test_window_gate(oracle_lib):
    """patches/0007:263-266 (miss window bookkeeping) and 414-429 (2-in-W)."""
    c = mk(oracle_lib, n_slots=1, admit_mode=2, admit_window=8)
    c.observe(0, [2])
    c.step()                          # empty slot: admitted without a gate decision
    c.observe(0, [4])
    c.step()                          # victim 2; 4 has one miss -> denied, no budget spent
    s = c.stats()
    assert (s["admit_ok"], s["admit_denied"], s["scheduled"]) == (0, 1, 1)
    g = c.gate_state(0)
    assert g["miss_prev"][4] == U64_MAX and g["miss_last"][4] == 1
    c.observe(0, [4])
    c.step()                          # second miss 1 step later -> admitted
    s = c.stats()
    assert (s["admit_ok"], s["admit_denied"], s["scheduled"]) == (1, 1, 2)
    assert c.tables(0)["expert_slot"][2] == -1


def test_window_gate_expires(oracle_lib):
    c = mk(oracle_lib, n_slots=1, admit_mode=2, admit_window=2)
    c.observe(0, [1]); c.step()
    c.observe(0, [5]); c.step()       # first miss of 5 at step 1
    for _ in range(3):
        c.step()                      # steps pass without 5
    c.observe(0, [5]); c.step()       # second miss 4 steps later: outside W=2
    assert c.stats()["admit_denied"] == 2 and c.stats()["admit_ok"] == 0


def test_heat_gate(oracle_lib):
    """patches/0007:422: admit iff heat[id] > 1.25 heat[victim] + floor."""
    c = mk(oracle_lib, n_slots=1, admit_mode=1, admit_floor=1.0, admit_half=64)
    c.observe(0, [1]); c.step()
    decided = []
    for tok in range(5):
        c.observe(0, [2])
        c.step()
        decided.append(c.stats()["admit_ok"])
    # heat[2] after k observations = k; heat[1] = 1: admitted once k > 2.25
    assert decided == [0, 0, 1, 1, 1]
    assert c.gate_state(0)["heat"][2] == 5.0


def test_heat_decay(oracle_lib):
    c = mk(oracle_lib, n_slots=1, admit_mode=1, admit_half=2)
    c.observe(0, [3]); c.observe(0, [3])
    c.step()                          # n_steps 1
    assert c.gate_state(0)["heat"][3] == 2.0
    c.step()                          # n_steps 2: halved
    assert c.gate_state(0)["heat"][3] == 1.0


def test_batches_are_not_observed(oracle_lib):
    """The observe callback returns early for batches (docs/EVICTION.md:147)."""
    c = mk(oracle_lib)
    c.observe(0, np.array([[1, 2], [3, 4]]))
    assert c.stats()["misses"] == 0
    c.observe(0, np.array([[1, 2]]))
    assert c.stats()["misses"] == 2


def test_freeze_schedules_nothing(oracle_lib):
    c = mk(oracle_lib, freeze=True)
    c.observe(0, [1, 2, 3])
    c.step()
    assert c.jobs().shape[0] == 0 and c.stats()["scheduled"] == 0


def test_prior_moves_with_table(oracle_lib):
    """patches/0007:326-348: prior[e] = delta iff the table maps e to a slot."""
    c = mk(oracle_lib, n_slots=2, cache_prior=0.01)
    c.observe(0, [4, 6]); c.step(); c.step()
    tbl, prior = c.dev_table(0)
    assert list(np.nonzero(tbl != 2)[0]) == [4, 6]
    assert np.allclose(prior[[4, 6]], 0.01) and prior.sum() == np.float32(0.02)


def test_batched_table_flush_counter(oracle_lib):
    c = mk(oracle_lib, batch_tables=True)
    c.step()
    assert c.stats()["table_flushes"] == 0
    c.observe(0, [1]); c.step(); c.step()
    assert c.stats()["table_flushes"] == 1     # only the publishing step is dirty


def test_early_issue_pool(oracle_lib):
    """patches/0006:251-293 and 843-913: uploads from the pre-freed pool during
    observation (lowest free slot first), pool topped up at the step."""
    c = mk(oracle_lib, n_slots=3, early_issue=True, max_inserts=2)
    c.observe(0, [5, 6, 7])           # budget 2 per call: 5 -> slot 0, 6 -> slot 1
    assert [tuple(r[:3]) for r in c.jobs()] == [(0, 5, 0), (0, 6, 1)]
    c.step()                          # publish; pool has 1 free (< 2): evict LRU -> slot 0
    t = c.tables(0)
    assert list(t["slot_expert"]) == [-1, 6, -1]
    assert c.stats()["uploads"] == 2


def test_spec_probation(oracle_lib):
    """patches/0007:660-668: a speculative upload is published with recency 1 and
    protected through the next step."""
    pred = lambda layer, cur, nprev, k: [3]
    c = oracle_lib.OracleCache(n_layers=2, n_expert=8, n_slots=3, max_inserts=1,
                               early_issue=True, predict_top=1, predictor=pred,
                               spec_probation=True)
    c.observe(0, [1])                 # demand: 1 -> layer 0; predicted 3 -> layer 1
    jobs = [tuple(r) for r in c.jobs()]
    assert (1, 3, 0, 1) in jobs
    c.step()
    t = c.tables(1)
    assert t["slot_expert"][0] == 3 and t["last_use"][0] == 1 and t["protect"][0] == 1


def test_map_text_format(oracle_lib):
    c = oracle_lib.OracleCache(n_layers=2, n_expert=8, n_slots=3, max_inserts=2)
    assert c.map_header() == "moe-map 1 2\nlayer 0 3 8\nlayer 1 3 8\n"
    c.observe(0, [4, 2]); c.observe(1, [7])
    c.step(); c.step()
    assert c.map_frame() == "step 2\nmap 0 2 4 -1\nmap 1 7 -1 -1\n"


def test_heat_file_round_trip_and_warm_start(oracle_lib, tmp_path):
    c = oracle_lib.OracleCache(n_layers=2, n_expert=8, n_slots=3, use_heat_counts=True)
    for _ in range(4):
        c.observe(0, [5, 1]); c.observe(1, [2])
    c.observe(0, [1, 6])
    path = str(tmp_path / "heat.txt")
    assert c.save_heat(path)
    text = open(path).read().splitlines()
    assert text[0] == "moe-heat 1 2 8"
    assert sorted(text[1:]) == sorted(["0 1 5", "0 5 4", "0 6 1", "1 2 4"])
    d = oracle_lib.OracleCache(n_layers=2, n_expert=8, n_slots=3, use_heat_counts=True)
    assert d.load_heat(path) == 4
    assert list(d.gate_state(0)["use_count"][[1, 5, 6]]) == [2, 2, 0]
    placed = d.warm_start()
    t = d.tables(0)
    # stable sort by count desc: 1 (2), 5 (2); 6 has 0 after halving -> not placed
    assert placed == 3 and list(t["slot_expert"]) == [1, 5, -1]
    assert list(t["last_use"][:2]) == [3, 2] and d.stats()["clock"] == 3
    wrong = oracle_lib.OracleCache(n_layers=3, n_expert=8, n_slots=3, use_heat_counts=True)
    assert wrong.load_heat(path) == -1
    assert not os.path.exists(path + ".tmp")


def test_slot_profile_sizes(oracle_lib):
    c = oracle_lib.OracleCache(n_layers=3, n_expert=16, n_slots=4, slot_profile=[2, 6, 4])
    assert [c.n_slots(L) for L in range(3)] == [2, 6, 4]
