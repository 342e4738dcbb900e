"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars (north_star): expert ids, routing weights, slot tables and admission
decisions bit-exact; layer outputs within relative L2 <= 1e-3 and max-abs
<= 1e-2 of the oracle (same Q8_1 activation quantisation).  The oracle's rows
follow the GEMV kernels' fp32 order, so the GEMV paths' outputs are also
asserted equal bit for bit; the double-accumulated rows stay the precision
reference (test_oracle.py).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import (MAX_ABS_TOL, REL_L2_TOL, ar1_states, assert_same_bits, check_decode_layer, rel_l2,
                      rms_norm)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8
Q4K, Q6K = 12, 14


def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def lib():
    _needs_gpu()
    from moe_prefetch_b200 import _lib
    return _lib.load()


def _p(t):
    return C.c_void_p(t.data_ptr())


def _s():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


# ---------------------------------------------------------------------------
# quantiser: device bytes == oracle bytes
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("qtype", [Q4K, Q6K])
def test_quantize_bit_identical(lib, oracle_lib, qtype):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(256 * 4096) * 0.02).astype(np.float32)
    x[:256] = 0.0                      # all-zero block
    x[256:512] = np.abs(x[256:512])    # all-positive block (min clamps to 0)
    bb = 144 if qtype == Q4K else 210
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(x.size // 256 * bb, dtype=torch.uint8, device="cuda")
    assert lib.moe_quantize(_p(xd), _p(yd), x.size, qtype, _s()) == 0
    torch.cuda.synchronize()
    ref = oracle_lib.quantize(x, qtype)
    assert np.array_equal(yd.cpu().numpy(), ref)


# ---------------------------------------------------------------------------
# router: bit-exact logits, ids, weights
# ---------------------------------------------------------------------------
def _router_case(lib, oracle_lib, W, X, k, table=None, ns=0, delta=0.0):
    n_tok, _ = X.shape
    n_exp = W.shape[0]
    Wd = torch.from_numpy(W).cuda()
    Xd = torch.from_numpy(X).cuda()
    ids = torch.empty(n_tok, k, dtype=torch.int32, device="cuda")
    w = torch.empty(n_tok, k, device="cuda")
    lg = torch.empty(n_tok, n_exp, device="cuda")
    td = torch.from_numpy(table).cuda() if table is not None else None
    rc = lib.moe_router_run(_p(Wd), _p(Xd), n_tok, n_exp, W.shape[1],
                            _p(td) if td is not None else None, ns, delta, k,
                            _p(ids), _p(w), _p(lg), _s())
    assert rc == 0
    torch.cuda.synchronize()
    ids, w, lg = ids.cpu().numpy(), w.cpu().numpy(), lg.cpu().numpy()
    for t in range(n_tok):
        prior = None
        if table is not None and delta > 0 and n_tok == 1:
            prior = np.where(table != ns, np.float32(delta), np.float32(0)).astype(np.float32)
        rid, rw, _, rlg = oracle_lib.router(W, X[t], k, prior)
        assert np.array_equal(lg[t].view(np.uint32), rlg.view(np.uint32)), f"logits token {t}"
        assert np.array_equal(ids[t], rid), f"ids token {t}: {ids[t]} vs {rid}"
        assert np.array_equal(w[t].view(np.uint32), rw.view(np.uint32)), f"weights token {t}"
    return ids


@pytest.mark.parametrize("n_exp", [128, 256])
def test_router_bit_exact(lib, oracle_lib, n_exp):
    rng = np.random.default_rng(11)
    W = (rng.standard_normal((n_exp, H)) * 0.02).astype(np.float32)
    X = rms_norm(rng.standard_normal((64, H)))
    _router_case(lib, oracle_lib, W, X, K)


@pytest.mark.parametrize("n_exp", [128, 256])
@pytest.mark.parametrize("n_tok", [1, 3, 4, 5, 32, 63, 64, 65, 200])
def test_batch_router_bit_exact(lib, oracle_lib, n_exp, n_tok):
    """Without a logits output the router runs as clusters of 8 CTAs: 4
    tokens per cluster up to 64 tokens, 8 above.  Ids and weights must equal
    the oracle's bit for bit for every shape, ragged last clusters included."""
    rng = np.random.default_rng(100 + n_tok)
    W = (rng.standard_normal((n_exp, H)) * 0.02).astype(np.float32)
    X = rms_norm(rng.standard_normal((n_tok, H)))
    Wd = torch.from_numpy(W).cuda()
    Xd = torch.from_numpy(X).cuda()
    ids = torch.empty(n_tok, K, dtype=torch.int32, device="cuda")
    w = torch.empty(n_tok, K, device="cuda")
    rc = lib.moe_router_run(_p(Wd), _p(Xd), n_tok, n_exp, H, None, 0, 0.0, K, _p(ids), _p(w), None, _s())
    assert rc == 0
    torch.cuda.synchronize()
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    for t in range(n_tok):
        rid, rw, _, _ = oracle_lib.router(W, X[t], K, None)
        assert np.array_equal(ids[t], rid), f"ids token {t}: {ids[t]} vs {rid}"
        assert np.array_equal(w[t].view(np.uint32), rw.view(np.uint32)), f"weights token {t}"


def test_router_ties_go_to_lower_id(lib, oracle_lib):
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    W[77] = W[12]            # identical rows -> identical logits
    W[100] = W[3]
    X = rms_norm(rng.standard_normal((8, H)))
    X[0] = 0.0               # all logits zero: ids must be 0..7
    ids = _router_case(lib, oracle_lib, W, X, K)
    assert list(ids[0]) == list(range(8))


def test_router_cache_prior(lib, oracle_lib):
    rng = np.random.default_rng(9)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    ns = 56
    changed = 0
    for t in range(32):
        X = rms_norm(rng.standard_normal((1, H)))
        table = np.full(E, ns, np.int32)
        res = rng.choice(E, ns, replace=False)
        table[res] = np.arange(ns, dtype=np.int32)
        a = _router_case(lib, oracle_lib, W, X, K, table, ns, 0.01)
        b = _router_case(lib, oracle_lib, W, X, K, None, ns, 0.0)
        changed += int(not np.array_equal(a, b))
    assert changed > 0, "delta=0.01 never changed a selection"


# ---------------------------------------------------------------------------
# one layer (config 0 shape), all experts resident
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def layer0(lib):
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=1)
    st.synth_resident(seed=7, keep_router=True)
    g, u, d = st.slot_views(0)
    W = st.routers[0].cpu().numpy()
    gate, up, down = (v[:E].cpu().numpy() for v in (g, u, d))
    yield st, W, gate, up, down
    st.close()


def _check_layer(y, ids, w, ry, rids, rw):
    assert np.array_equal(ids, rids)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert rel_l2(y, ry) <= REL_L2_TOL, rel_l2(y, ry)
    assert np.abs(y - ry).max() <= MAX_ABS_TOL
    assert_same_bits(y, ry, "layer output")


def test_layer_forward_batch1(layer0, oracle_lib):
    st, W, gate, up, down = layer0
    X = rms_norm(np.random.default_rng(12345).standard_normal((64, H)))
    ys, idss, ws = [], [], []
    for t in range(64):
        y, ids, w = st.layer_forward(0, torch.from_numpy(X[t:t + 1]).cuda())
        ys.append(y.cpu().numpy()[0]); idss.append(ids.cpu().numpy()[0]); ws.append(w.cpu().numpy()[0])
    st.sync()
    rids, rw, ry = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K)
    _check_layer(np.array(ys), np.array(idss), np.array(ws), ry, rids, rw)


def test_layer_forward_batched(layer0, oracle_lib):
    st, W, gate, up, down = layer0
    X = rms_norm(np.random.default_rng(99).standard_normal((32, H)))
    y, ids, w = st.layer_forward(0, torch.from_numpy(X).cuda())
    st.sync()
    rids, rw, ry = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K)
    _check_layer(y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), ry, rids, rw)


def _per_pair(st, x):
    """The per-pair kernels (one read of an expert's rows per routed pair),
    reached through the allocation-free entry point, which keeps them."""
    y = torch.empty_like(x)
    ids = torch.empty(x.shape[0], K, dtype=torch.int32, device=x.device)
    w = torch.empty(x.shape[0], K, device=x.device)
    st.layer_forward_noalloc(0, x, y, ids, w)
    return y, ids, w


@pytest.mark.parametrize("n_tok", [2, 9, 33, 170])
def test_grouped_batch_bit_identical_to_per_pair(layer0, n_tok):
    """n_tok > 1 groups the pairs by expert (one weight read per expert tile);
    the result must equal the per-pair kernels bit for bit, including past
    the grouping kernel's 1024-pair chunk (170 tokens = 1360 pairs)."""
    st = layer0[0]
    X = torch.from_numpy(rms_norm(np.random.default_rng(500 + n_tok).standard_normal((n_tok, H)))).cuda()
    y, ids, w = st.layer_forward(0, X)
    y1, ids1, w1 = _per_pair(st, X)
    st.sync()
    assert torch.equal(ids, ids1) and torch.equal(w.view(torch.int32), w1.view(torch.int32))
    assert torch.equal(y.view(torch.int32), y1.view(torch.int32))


def test_grouped_batch_skewed_routing(layer0, oracle_lib):
    """Every token identical: all pairs land on the same 8 experts, 64 pairs
    each, i.e. 8 tiles per expert and 120 idle experts."""
    st, W, gate, up, down = layer0
    x1 = rms_norm(np.random.default_rng(77).standard_normal((1, H)))
    X = np.repeat(x1, 64, axis=0)
    y, ids, w = st.layer_forward(0, torch.from_numpy(X).cuda())
    y1, _, _ = _per_pair(st, torch.from_numpy(X).cuda())
    st.sync()
    assert torch.equal(y.view(torch.int32), y1.view(torch.int32))
    rids, rw, ry = oracle_lib.moe_layer(X[:1], W, gate, up, down, Q6K, I, K)
    _check_layer(y.cpu().numpy()[:1], ids.cpu().numpy()[:1], w.cpu().numpy()[:1], ry, rids, rw)
    assert (y.cpu().numpy() == y.cpu().numpy()[:1]).all()


def test_layer_forward_vs_fp32_and_q8K_informational(layer0, oracle_lib):
    """How far the Q8_1 kernel is from a plain fp32 reference and from the
    ggml CPU path's Q8_K activations (informational bounds, not the bar)."""
    st, W, gate, up, down = layer0
    X = rms_norm(np.random.default_rng(1).standard_normal((4, H)))
    y, ids, w = st.layer_forward(0, torch.from_numpy(X).cuda())
    y = y.cpu().numpy()
    _, _, ry8k = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K, path="q8K")
    assert rel_l2(y, ry8k) < 0.05


# ---------------------------------------------------------------------------
# decode stack: persistent kernel
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def stack4(lib):
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=4)
    st.synth_resident(seed=21, keep_router=True)
    yield st
    st.close()


def test_decode_stack_parity(stack4, oracle_lib):
    st = stack4
    n_tok = 6
    h = ar1_states(n_tok, H, seed=4)
    out, dm = st.decode(torch.from_numpy(h).cuda(), debug=True)
    st.sync()
    out = out.cpu().numpy()
    dumps = {k: v.cpu().numpy() for k, v in dm.items()}
    grid = st.decode_info()["grid"]
    for L in range(st.n_layers):
        g, u, d = st.slot_views(L)
        gate, up, down = (v[:E].cpu().numpy() for v in (g, u, d))
        W = st.routers[L].cpu().numpy()
        for t in range(n_tok):
            check_decode_layer(oracle_lib, h[t], dumps, t, L, W, gate, up, down, grid)
    # residual stream: out = h + y_0 + ... + y_{L-1} in fp32, in that order
    ys = dumps["y"]
    r = h.copy()
    for L in range(st.n_layers):
        r = (r + ys[:, L]).astype(np.float32)
    assert np.array_equal(out.view(np.uint32), r.view(np.uint32))
    # router inputs are the RMS-normed residual
    r = h.copy()
    for L in range(st.n_layers):
        assert rel_l2(dumps["x"][:, L], rms_norm(r, 1e-6)) < 1e-5
        r = (r + ys[:, L]).astype(np.float32)


def test_decode_prefetch_invariant(stack4):
    """The persistent kernel prefetches into L2, for the next layer, the
    experts the previous token used there.  That may change when bytes move,
    never the result: one launch over 8 tokens (prefetch hits and misses)
    gives the same bits as 8 one-token launches (no prefetch at all)."""
    st = stack4
    h = torch.from_numpy(ar1_states(8, H, seed=12)).cuda()
    out = st.decode(h)
    for t in range(8):
        assert torch.equal(st.decode(h[t:t + 1].contiguous()), out[t:t + 1])
    st.sync()


def test_decode_early_copies_invariant(stack4, oracle_lib):
    """With the cache prior off, the persistent kernel requests the gate/up
    rows of the logits' top-k before the exact selection is known, and
    requests them again for any rank whose exact id differs.  That changes
    when bytes move, never the result: early copies (default), no early
    copies, and early copies with a wrong rank-0 prediction in every other
    (token, layer), so that half of the layers take the re-issue path, give
    the same outputs and dumps bit for bit, and match the oracle."""
    st = stack4
    n_tok = 5
    h = ar1_states(n_tok, H, seed=31)
    hd = torch.from_numpy(h).cuda()
    runs = [st.decode(hd, debug=True, spec=m) for m in (0, 1, 2)]
    st.sync()
    out0, dm0 = runs[0]
    for out, dm in runs[1:]:
        assert torch.equal(out, out0)
        for key in ("x", "ids", "w", "y"):
            assert torch.equal(dm[key], dm0[key]), key
    dumps = {k: v.cpu().numpy() for k, v in runs[2][1].items()}
    grid = st.decode_info()["grid"]
    for L in range(st.n_layers):
        g, u, d = st.slot_views(L)
        gate, up, down = (v[:E].cpu().numpy() for v in (g, u, d))
        W = st.routers[L].cpu().numpy()
        for t in range(n_tok):
            check_decode_layer(oracle_lib, h[t], dumps, t, L, W, gate, up, down, grid)


def test_decode_matches_layer_forward(stack4):
    """Same x and same routed experts -> the persistent kernel and the
    stand-alone kernels give the same output bits (same unit mapping, same
    reduction order).  Their routers sum the logits in different canonical
    orders, so the ids agree except at exact near-ties."""
    st = stack4
    h = ar1_states(4, H, seed=8)
    out, dm = st.decode(torch.from_numpy(h).cuda(), debug=True)
    xs, ys = dm["x"], dm["y"]
    same = 0
    for L in range(st.n_layers):
        for t in range(4):
            y, ids, w = st.layer_forward(L, xs[t, L:L + 1].contiguous())
            if torch.equal(ids[0], dm["ids"][t, L]):
                same += 1
                if torch.equal(w[0], dm["w"][t, L]):
                    assert torch.equal(y[0], ys[t, L])
    st.sync()
    assert same >= 15


def test_decode_host_e2e(stack4):
    st = stack4
    h = ar1_states(5, H, seed=6)
    ref = st.decode(torch.from_numpy(h).cuda()).cpu()
    hp = torch.from_numpy(h).pin_memory()
    op = torch.empty_like(hp).pin_memory()
    st.decode_host(hp, op)
    assert torch.equal(ref, op)


# ---------------------------------------------------------------------------
# misses: experts not resident are read zero-copy from the host weights
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def miss_stack(lib, layer0):
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    _, W, gate, up, down = layer0
    st = MoeStack(n_layers=2, cache=MoeCacheConfig(n_slots=40))
    hg = torch.from_numpy(gate.copy()).pin_memory()
    hu = torch.from_numpy(up.copy()).pin_memory()
    hd = torch.from_numpy(down.copy()).pin_memory()
    Wd = torch.from_numpy(W).cuda()
    for L in range(2):
        st.set_router(L, Wd)
        st.set_expert_weights(L, hg, hu, hd)
        rng = np.random.default_rng(L)
        se = rng.choice(E, 40, replace=False).astype(np.int32)
        st.place(L, se, copy=True)
    yield st, W, gate, up, down
    st.close()


def test_layer_forward_with_misses(miss_stack, oracle_lib):
    st, W, gate, up, down = miss_stack
    X = rms_norm(np.random.default_rng(77).standard_normal((8, H)))
    y, ids, w = st.layer_forward(0, torch.from_numpy(X).cuda())
    st.sync()
    rids, rw, ry = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K)
    _check_layer(y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), ry, rids, rw)


@pytest.mark.parametrize("spec", [0, 2])
def test_decode_with_misses(miss_stack, oracle_lib, spec):
    """spec 2: every other (token, layer) re-issues its gate/up copies after
    a wrong prediction, with missed experts among the ranks."""
    st, W, gate, up, down = miss_stack
    h = ar1_states(4, H, seed=10)
    out, dm = st.decode(torch.from_numpy(h).cuda(), debug=True, spec=spec)
    st.sync()
    dumps = {k: v.cpu().numpy() for k, v in dm.items()}
    ids = dumps["ids"]
    tabs = [st.tables(L)["expert_slot"] for L in range(2)]
    n_miss = sum(int((tabs[L][ids[:, L]] < 0).sum()) for L in range(2))
    assert n_miss > 0, "placement produced no misses"
    grid = st.decode_info()["grid"]
    for L in range(2):
        for t in range(h.shape[0]):
            check_decode_layer(oracle_lib, h[t], dumps, t, L, W, gate, up, down, grid)
