"""Device slot table vs the oracle's restatement of llama-moecache.cpp
(patches 0006/0007/0008): tables, recency, in-flight flags, admission
decisions and counters bit-exact after every step; uploaded slot bytes equal
the host expert bytes the table says they hold."""
import numpy as np
import pytest

from conftest import ar1_states, check_decode_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H = 2048


def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _trace(n_tok, n_layers, n_expert, k, seed, keep=5):
    """Routing with locality: each layer keeps most of the previous token's
    experts and draws the rest from a skewed distribution."""
    rng = np.random.default_rng(seed)
    pop = rng.permutation(n_expert)
    p = 1.0 / np.arange(1, n_expert + 1) ** 1.1
    p /= p.sum()
    prev = [list(rng.choice(n_expert, k, replace=False)) for _ in range(n_layers)]
    out = np.zeros((n_tok, n_layers, k), np.int32)
    for t in range(n_tok):
        for L in range(n_layers):
            cur = list(rng.permutation(prev[L])[:keep])
            while len(cur) < k:
                e = int(pop[rng.choice(n_expert, p=p)])
                if e not in cur:
                    cur.append(e)
            rng.shuffle(cur)
            out[t, L] = cur
            prev[L] = cur
    return out


def _compare(st, oc, n_layers, ctx=""):
    for L in range(n_layers):
        d = st.tables(L)
        o = oc.tables(L)
        for key in ("expert_slot", "slot_expert", "last_use", "in_flight", "protect"):
            assert np.array_equal(d[key], o[key]), f"{ctx} layer {L} {key}:\n{d[key]}\n{o[key]}"
        gd, go = st.gate_state(L), oc.gate_state(L)
        for key in ("heat", "miss_last", "miss_prev"):
            assert np.array_equal(gd[key], go[key]), f"{ctx} layer {L} {key}"
    sd, so = st.stats(), oc.stats()
    for key in ("steps", "clock", "hits", "misses", "scheduled", "copied", "published",
                "admit_ok", "admit_denied", "table_flushes"):
        assert sd[key] == so[key], f"{ctx} stat {key}: {sd[key]} vs {so[key]}"


def _host_weights(n_expert, gate_bytes, down_bytes, seed):
    rng = np.random.default_rng(seed)
    mk = lambda n: torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8)).pin_memory()
    return mk(n_expert * gate_bytes), mk(n_expert * gate_bytes), mk(n_expert * down_bytes)


@pytest.mark.parametrize("admit,max_inserts,batch,profile", [
    ("off", 2, True, None),
    ("window", 2, True, [6, 8, 12]),
    ("heat", 3, False, None),
    ("window", 1, False, [8, 5, 8]),
])
def test_slot_table_matches_oracle(oracle_lib, admit, max_inserts, batch, profile):
    _needs_gpu()
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack, format_slot_profile
    L, E, k, n_ff = 3, 32, 8, 256
    cfg = MoeCacheConfig(n_slots=10, max_inserts=max_inserts, admit=admit,
                         batch_tables=batch, admit_half=16,
                         slot_profile=format_slot_profile(profile) if profile else "")
    st = MoeStack(n_layers=L, n_expert=E, n_used=k, n_ff=n_ff, cache=cfg)
    hw = [_host_weights(E, st.gate_bytes, st.down_bytes, s) for s in range(L)]
    for il in range(L):
        st.set_expert_weights(il, *hw[il])
    oc = oracle_lib.OracleCache(L, E, 10, slot_profile=st.ns, max_inserts=max_inserts,
                                admit_mode=cfg.admit_mode, admit_window=cfg.admit_window,
                                admit_half=16, admit_floor=cfg.admit_floor,
                                batch_tables=batch)
    tr = _trace(40, L, E, k, seed=hash((admit, max_inserts)) & 0xFFFF)
    for t in range(tr.shape[0]):
        for il in range(L):
            ids = torch.from_numpy(tr[t, il]).cuda()
            st.observe(il, ids)
            oc.observe(il, tr[t, il])
        st.step()
        oc.step()
        _compare(st, oc, L, f"token {t}")
    # every published slot holds the bytes of its expert
    st.step(); oc.step()
    torch.cuda.synchronize()
    for il in range(L):
        g, u, d = st.slot_views(il)
        se = st.tables(il)["slot_expert"]
        hg, hu, hd = (x.numpy() for x in hw[il])
        for s, e in enumerate(se):
            if e < 0:
                continue
            assert np.array_equal(g[s].cpu().numpy(), hg[e * st.gate_bytes:(e + 1) * st.gate_bytes])
            assert np.array_equal(d[s].cpu().numpy(), hd[e * st.down_bytes:(e + 1) * st.down_bytes])
    st.close()


def _decode_with_cache(oracle_lib, L, n_tok, ns, profile=None, prior=0.01, seed=33, early=False):
    """Batch-1 decode token by token through a constrained cache: misses
    served zero-copy, second-miss (window) admission, uploads on the copy
    stream, deterministic publication.  After every step the device tables
    equal the oracle's (fed the same routed ids), and every layer's ids and
    weights are bit-exact and its output within tolerance, with the router's
    prior taken from the oracle's published table."""
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack, format_slot_profile
    E, k = 128, 8
    # weights: generate resident on a helper stack, then host copies
    src = MoeStack(n_layers=L)
    src.synth_resident(seed=seed, keep_router=True)
    host = []
    for il in range(L):
        g, u, d = src.slot_views(il)
        host.append(tuple(v[:E].contiguous().cpu().pin_memory() for v in (g, u, d)))
    routers = [r.clone() for r in src.routers]
    src.close()
    torch.cuda.synchronize()
    cfg = MoeCacheConfig(n_slots=ns, max_inserts=2, admit="window", batch_tables=True,
                         cache_prior=prior, early_issue=early,
                         slot_profile=format_slot_profile(profile) if profile else "")
    st = MoeStack(n_layers=L, cache=cfg)
    for il in range(L):
        st.set_router(il, routers[il])
        st.set_expert_weights(il, *host[il])
    oc = oracle_lib.OracleCache(L, E, ns, slot_profile=st.ns, max_inserts=2, admit_mode=2,
                                batch_tables=True, cache_prior=prior, early_issue=early)
    h = ar1_states(n_tok, H, seed=2)
    grid = st.decode_info()["grid"]
    for t in range(h.shape[0]):
        out, dm = st.decode(torch.from_numpy(h[t:t + 1]).cuda(), debug=True)
        st.sync()
        dumps = {q: v.cpu().numpy() for q, v in dm.items()}
        for il in range(L):
            tbl, pri = oc.dev_table(il)
            W = routers[il].cpu().numpy()
            gate, up, down = (x.numpy().reshape(E, -1) for x in host[il])
            check_decode_layer(oracle_lib, h[t], dumps, 0, il, W, gate, up, down, grid,
                               prior=pri)
            oc.observe(il, dumps["ids"][0, il])
        st.step()
        oc.step()
        _compare(st, oc, L, f"token {t}")
    s = st.stats()
    assert s["misses"] > 0 and s["scheduled"] > 0 and s["published"] > 0
    st.close()
    return s


def test_decode_with_cache_end_to_end(oracle_lib):
    """The config-2 flow at small scale: 2 layers, 24 slots, 24 tokens."""
    _needs_gpu()
    _decode_with_cache(oracle_lib, L=2, n_tok=24, ns=24)


def test_decode_with_cache_config2_scale(oracle_lib):
    """The config-2 flow at its own scale: 128 experts, a 56-slot budget
    spread over 8 layers by the byte-priced greedy allocation (grid 16 / 32 /
    56 / 96), delta = 0.01, window admission, batched tables, 64 tokens."""
    _needs_gpu()
    from moe_prefetch_b200 import greedy_allocate_bytes
    L = 8
    grid = [16, 32, 56, 96]
    # per-layer miss curves (misses per 8 routed ids at each grid size):
    # layers differ in how much a slot helps, so the greedy spreads the budget
    rng = np.random.default_rng(5)
    scale = rng.uniform(0.5, 2.0, L)
    miss8 = {n: [float(8 * scale[il] * (1 - n / 128) ** (1 + il % 3)) for il in range(L)] for n in grid}
    caps, used, budget = greedy_allocate_bytes(miss8, grid, L, 56, [], [3059712] * L)
    assert used <= budget and len(set(caps)) > 1
    s = _decode_with_cache(oracle_lib, L=L, n_tok=64, ns=56, profile=caps, seed=44)
    assert s["hits"] > 0 and s["copied"] > 0


def _cached_pair(tmp_path, seed=61, L=3, ns=20):
    """A stack with a constrained cache over host weights (misses zero-copy,
    uploads on the copy stream), plus the host weights and routers to build
    another one with the same weights."""
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    E = 128
    src = MoeStack(n_layers=L)
    src.synth_resident(seed=seed, keep_router=True)
    host = []
    for il in range(L):
        g, u, d = src.slot_views(il)
        host.append(tuple(v[:E].contiguous().cpu().pin_memory() for v in (g, u, d)))
    routers = [r.clone() for r in src.routers]
    src.close()
    torch.cuda.synchronize()

    def make(**kw):
        args = dict(n_slots=ns, max_inserts=2, admit="window", batch_tables=True, cache_prior=0.01)
        args.update(kw)
        cfg = MoeCacheConfig(**args)
        st = MoeStack(n_layers=L, cache=cfg)
        for il in range(L):
            st.set_router(il, routers[il])
            st.set_expert_weights(il, *host[il])
        return st
    return make


def _run_tokens(st, h):
    outs, tabs = [], []
    for t in range(h.shape[0]):
        outs.append(st.decode(torch.from_numpy(h[t:t + 1]).cuda()).cpu().numpy())
        st.step()
        st.sync()
        tabs.append([st.tables(il)["expert_slot"].copy() for il in range(st.n_layers)])
    return np.concatenate(outs), tabs


def test_map_record_replay_reproduces_tables_and_outputs(tmp_path):
    """LLAMA_MOE_MAP_RECORD writes the published placement after every step;
    a stack with LLAMA_MOE_MAP_REPLAY of that file (and a different insert
    budget of its own) reproduces every step's tables and every output bit
    for bit (patches/0008:417-518).  LLAMA_MOE_ROUTE_TRACE lines carry the
    routed ids and the slots the router saw."""
    _needs_gpu()
    make = _cached_pair(tmp_path)
    rec, trace = str(tmp_path / "map.txt"), str(tmp_path / "route.txt")
    h = ar1_states(20, H, seed=9)
    st = make(map_record=rec, route_trace=trace)
    out_a, tabs_a = _run_tokens(st, h)
    s_a = st.stats()
    st.close()
    assert s_a["published"] > 0 and s_a["misses"] > 0
    lines = open(rec).read().splitlines()
    assert lines[0] == "moe-map 1 3" and lines[1] == "layer 0 20 128"
    assert sum(1 for ln in lines if ln.startswith("step ")) == 21          # step 0 .. 20
    routes = open(trace).read().splitlines()
    assert len(routes) == 20 * 3
    f = routes[4].split()                                                 # token 1, layer 1
    assert f[:5] == ["route", "1", "1", "8", "1"] and len(f) == 5 + 8
    assert all(int(p.split(":")[0]) in range(128) and int(p.split(":")[1]) in range(-1, 20) for p in f[5:])
    # replay with another budget of its own: the frames decide the placement
    st = make(map_replay=rec, max_inserts=1)
    out_b, tabs_b = _run_tokens(st, h)
    st.close()
    assert np.array_equal(out_a.view(np.uint32), out_b.view(np.uint32))
    for ta, tb in zip(tabs_a, tabs_b):
        for a, b in zip(ta, tb):
            assert np.array_equal(a, b)
    # a frame that does not match the stack is refused
    from moe_prefetch_b200._lib import MoeError
    bad = str(tmp_path / "bad.txt")
    with open(bad, "w") as fh:
        fh.write("moe-map 1 2\nlayer 0 20 128\nlayer 1 20 128\n")
    st = make(map_replay=bad)
    with pytest.raises(MoeError):
        st.decode(torch.from_numpy(h[:1]).cuda())
    st.close()


def test_heat_file_saved_every_512_steps_and_warm_starts(tmp_path):
    """LLAMA_MOE_HEAT_FILE: the routed-use counts go to the file every 512
    steps (patches/0007:749-753), and a new stack places the hottest experts
    before its first token (0007:567-618): the counts halved on load, the
    hottest in slot 0, never-routed experts left out."""
    _needs_gpu()
    from moe_prefetch_b200.stack import load_heat
    make = _cached_pair(tmp_path, L=2, ns=6)
    path = str(tmp_path / "heat.txt")
    st = make(heat_file=path)
    hot = [[5, 9, 17, 33, 40, 64, 70, 99], [1, 2, 3, 4, 5, 6, 7, 8]]
    for step in range(512):
        for il in range(2):
            ids = torch.tensor(hot[il] if step % 2 == 0 else hot[il][:4], dtype=torch.int32, device="cuda")
            st.observe(il, ids)
        st.step()
    st.sync()
    st.close()
    counts = load_heat(path, 2, 128)
    assert counts is not None
    assert counts[0, 5] == 512 // 2 and counts[0, 40] == 256 // 2 and counts[0, 6] == 0
    st = make(heat_file=path)
    st.start()
    for il in range(2):
        se = st.tables(il)["slot_expert"]
        assert list(se[:4]) == hot[il][:4]                    # 512 uses each, in id order
        assert set(se[4:6]) <= set(hot[il][4:]) and (se >= 0).all()
    st.close()


@pytest.mark.parametrize("admit,predict,probation", [
    ("off", False, False),
    ("window", False, False),
    ("heat", True, False),
    ("window", True, True),
    ("off", True, True),
])
def test_early_issue_matches_oracle(oracle_lib, admit, predict, probation):
    """LLAMA_MOE_EARLY_ISSUE (patches/0006:251-293, :843-913; 0007:230-321):
    admitted misses take slots of a free pool when the layer is observed,
    the step publishes them and refills the pool; with a predictor hook its
    ids for the next layer become speculative uploads (probation with
    LLAMA_MOE_SPEC_PROBATION).  Tables, recency, flags and counters equal the
    oracle's after every step; every published slot holds its expert's
    bytes."""
    _needs_gpu()
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    L, E, k, n_ff, ns = 3, 32, 8, 256, 12
    cfg = MoeCacheConfig(n_slots=ns, max_inserts=2, admit=admit, batch_tables=True, admit_half=16,
                         early_issue=True, predict_top=3, spec_probation=probation)
    st = MoeStack(n_layers=L, n_expert=E, n_used=k, n_ff=n_ff, cache=cfg)
    hw = [_host_weights(E, st.gate_bytes, st.down_bytes, 40 + s) for s in range(L)]
    for il in range(L):
        st.set_expert_weights(il, *hw[il])
    calls = []

    def pred(layer, cur, next_prev, kk):
        calls.append(layer)
        return (list(next_prev) + [(v + 1) % E for v in cur])[:kk]
    if predict:
        st.set_predictor(pred)
    oc = oracle_lib.OracleCache(L, E, ns, max_inserts=2, admit_mode=cfg.admit_mode,
                                admit_window=cfg.admit_window, admit_half=16,
                                admit_floor=cfg.admit_floor, batch_tables=True, spec_probation=probation,
                                early_issue=True, predict_top=3, predictor=pred if predict else None)
    seen = []
    st.set_observe_hook(lambda layer, ids: seen.append((layer, ids.tolist())))
    tr = _trace(40, L, E, k, seed=hash((admit, predict, probation)) & 0xFFFF)
    for t in range(tr.shape[0]):
        for il in range(L):
            st.observe(il, torch.from_numpy(tr[t, il]).cuda())
            oc.observe(il, tr[t, il])
        st.step()
        oc.step()
        _compare(st, oc, L, f"token {t}")
        assert st.stats()["uploads"] == oc.stats()["uploads"], f"token {t}: uploads"
    assert st.stats()["uploads"] > 0
    assert [x[0] for x in seen] == [il for _ in range(tr.shape[0]) for il in range(L)]
    assert seen[4] == (1, [tr[1, 1].tolist()])
    if predict:
        assert len(calls) == 2 * tr.shape[0] * (L - 1)    # device stack and oracle, layers with a next one
    st.step(); oc.step()
    torch.cuda.synchronize()
    for il in range(L):
        g, u, d = st.slot_views(il)
        se = st.tables(il)["slot_expert"]
        hg, hu, hd = (x.numpy() for x in hw[il])
        for sl, e in enumerate(se):
            if e >= 0:
                assert np.array_equal(g[sl].cpu().numpy(), hg[e * st.gate_bytes:(e + 1) * st.gate_bytes])
                assert np.array_equal(d[sl].cpu().numpy(), hd[e * st.down_bytes:(e + 1) * st.down_bytes])
    st.close()


def test_decode_with_cache_early_issue(oracle_lib):
    """The persistent decode kernel's own observation with early issue: the
    admitted misses take pool slots inside the launch, the step publishes
    them; tables equal the oracle's and outputs are bit-exact every step."""
    _needs_gpu()
    s = _decode_with_cache(oracle_lib, L=3, n_tok=24, ns=24, early=True)
    assert s["uploads"] > 0


@pytest.mark.parametrize("early,admit,predict", [
    (False, "off", False),
    (False, "window", False),
    (True, "off", False),
    (True, "heat", True),
])
def test_evictor_matches_oracle(oracle_lib, early, admit, predict):
    """LLAMA_MOE_EVICTOR (patches/0006:402-426, :790-913; 0007:680-727): the
    device scores each layer with the model at every step and evicts the
    lowest score (recency breaking ties) in the scheduling and the early-issue
    top-up; layer 1 has no model and keeps LRU.  Tables, recency, flags and
    counters equal the oracle's after every step; every published slot holds
    its expert's bytes."""
    _needs_gpu()
    from conftest import toy_moep
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    L, E, k, n_ff, ns = 3, 32, 8, 256, 12
    model = toy_moep(L, E, [0, 2], seed=17, prior=0.25)
    cfg = MoeCacheConfig(n_slots=ns, max_inserts=2, admit=admit, batch_tables=True, admit_half=16,
                         early_issue=early, predict_top=3)
    st = MoeStack(n_layers=L, n_expert=E, n_used=k, n_ff=n_ff, cache=cfg)
    hw = [_host_weights(E, st.gate_bytes, st.down_bytes, 70 + s) for s in range(L)]
    for il in range(L):
        st.set_expert_weights(il, *hw[il])
    st.set_evictor(model)

    def pred(layer, cur, next_prev, kk):
        return (list(next_prev) + [(v + 3) % E for v in cur])[:kk]
    if predict:
        st.set_predictor(pred)
    oc = oracle_lib.OracleCache(L, E, ns, max_inserts=2, admit_mode=cfg.admit_mode,
                                admit_window=cfg.admit_window, admit_half=16, admit_floor=cfg.admit_floor,
                                batch_tables=True, early_issue=early, predict_top=3,
                                predictor=pred if predict else None)
    oc.set_evictor(model)
    tr = _trace(40, L, E, k, seed=hash((early, admit, predict, 3)) & 0xFFFF)
    lru = oracle_lib.OracleCache(L, E, ns, max_inserts=2, admit_mode=cfg.admit_mode,
                                 admit_window=cfg.admit_window, admit_half=16, admit_floor=cfg.admit_floor,
                                 batch_tables=True, early_issue=early, predict_top=3,
                                 predictor=pred if predict else None)
    differs = 0
    for t in range(tr.shape[0]):
        for il in range(L):
            st.observe(il, torch.from_numpy(tr[t, il]).cuda())
            oc.observe(il, tr[t, il])
            lru.observe(il, tr[t, il])
        st.step()
        oc.step()
        lru.step()
        _compare(st, oc, L, f"token {t}")
        differs += int(any(not np.array_equal(oc.tables(il)["slot_expert"], lru.tables(il)["slot_expert"])
                           for il in (0, 2)))
        assert np.array_equal(oc.tables(1)["slot_expert"], lru.tables(1)["slot_expert"]), "layer 1 keeps LRU"
    assert differs > 0, "the model never chose another victim than LRU"
    st.step(); oc.step()
    torch.cuda.synchronize()
    for il in range(L):
        g, u, d = st.slot_views(il)
        se = st.tables(il)["slot_expert"]
        hg, hu, hd = (x.numpy() for x in hw[il])
        for sl, e in enumerate(se):
            if e >= 0:
                assert np.array_equal(g[sl].cpu().numpy(), hg[e * st.gate_bytes:(e + 1) * st.gate_bytes])
                assert np.array_equal(d[sl].cpu().numpy(), hd[e * st.down_bytes:(e + 1) * st.down_bytes])
    st.set_evictor(None)
    st.close()
    oc.close()
    lru.close()
