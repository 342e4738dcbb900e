"""Just-in-time expert streaming (LLAMA_MOE_STREAM, patches/0010:951-1010,
its mover and cpp/llama-moe-planner.h) through the per-layer entry point.

After each single-token layer the lookahead of the next two layers' routers
claims pool slots for their best non-resident experts; the mover sends them
earliest deadline first in chunks on the copy stream and writes each one's
table word after its last byte.  The checks:

- outputs, ids and weights bit-identical to a stack without streaming (a
  routed expert reads the same bytes from its slot or from host memory);
- streamed experts reach their layer in time (found resident) on a workload
  whose layers leave the copies time to land;
- after the steps, tables are consistent (slot -> expert and expert -> slot
  agree, nothing in flight) and every resident slot holds its expert's bytes;
- with the cache prior, routing sees published residency only: every
  layer's ids and weights equal the oracle router's with the prior taken
  from the slots published at the last step, whatever landed since.
"""
import numpy as np
import pytest

from conftest import ar1_states

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, E, K = 2048, 128, 8


def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def weights():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    L = 4
    src = MoeStack(n_layers=L)
    src.synth_resident(seed=71, keep_router=True)
    host = []
    for il in range(L):
        g, u, d = src.slot_views(il)
        host.append(tuple(v[:E].contiguous().cpu().pin_memory() for v in (g, u, d)))
    routers = [r.clone() for r in src.routers]
    src.close()
    torch.cuda.synchronize()
    return L, host, routers


def _make(weights, **kw):
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    L, host, routers = weights
    args = dict(n_slots=40, max_inserts=2, admit="off", batch_tables=True, early_issue=True)
    args.update(kw)
    st = MoeStack(n_layers=L, cache=MoeCacheConfig(**args))
    for il in range(L):
        st.set_router(il, routers[il])
        st.set_expert_weights(il, *host[il])
    return st


def _next_input(x, y):
    """The next layer's input: RMS-normed residual sum (deterministic)."""
    z = x + y
    return z * torch.rsqrt((z * z).mean(-1, keepdim=True) + 1e-6)


def _run(st, h, per_layer=None, pause_s=0.0):
    """Token by token, layer by layer; per_layer(t, il, x, y, ids, w) sees
    every layer.  pause_s stands for the rest of a transformer layer
    (attention), during which copies land."""
    import time
    outs = []
    for t in range(h.shape[0]):
        x = torch.from_numpy(h[t:t + 1]).cuda()
        for il in range(st.n_layers):
            y, ids, w = st.layer_forward(il, x)
            if per_layer is not None:
                per_layer(t, il, x, y, ids, w)
            outs.append((y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()))
            x = _next_input(x, y)
            if pause_s:
                torch.cuda.synchronize()
                time.sleep(pause_s)
        st.step()
    return outs


def _check_consistent(st, host):
    torch.cuda.synchronize()
    for il in range(st.n_layers):
        tb = st.tables(il)
        es, se = tb["expert_slot"], tb["slot_expert"]
        assert not tb["in_flight"].any(), f"layer {il}: slots still in flight after the step"
        for e in range(E):
            if es[e] >= 0:
                assert se[es[e]] == e, f"layer {il}: expert {e} -> slot {es[e]} -> {se[es[e]]}"
        for s, e in enumerate(se):
            if e >= 0:
                assert es[e] == s, f"layer {il}: slot {s} -> expert {e} -> slot {es[e]}"
        g, u, d = st.slot_views(il)
        hg, hu, hd = (x.numpy().reshape(-1) for x in host[il])
        gb, db = st.gate_bytes, st.down_bytes
        for s, e in enumerate(se):
            if e >= 0:
                assert np.array_equal(g[s].cpu().numpy(), hg[e * gb:(e + 1) * gb]), f"layer {il} slot {s} gate"
                assert np.array_equal(u[s].cpu().numpy(), hu[e * gb:(e + 1) * gb]), f"layer {il} slot {s} up"
                assert np.array_equal(d[s].cpu().numpy(), hd[e * db:(e + 1) * db]), f"layer {il} slot {s} down"


def test_stream_bit_identical_and_in_time(weights):
    """Streaming changes when experts become resident, never what a layer
    computes; with a pause per layer the streamed experts arrive in time."""
    _needs_gpu()
    L, host, _ = weights
    h = ar1_states(24, H, seed=5)
    plain = _make(weights)
    ref = _run(plain, h, pause_s=0.0005)
    hits_plain = plain.stats()["hits"]
    plain.close()
    st = _make(weights, stream=True, stream_per_layer=4, stream_reserve=3)
    got = _run(st, h, pause_s=0.0005)
    for i, ((y0, i0, w0), (y1, i1, w1)) in enumerate(zip(ref, got)):
        tok, il = divmod(i, L)
        assert np.array_equal(i0, i1), f"token {tok} layer {il}: ids"
        assert np.array_equal(w0.view(np.uint32), w1.view(np.uint32)), f"token {tok} layer {il}: weights"
        assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32)), f"token {tok} layer {il}: output"
    ss = st.stream_stats()
    s = st.stats()
    assert ss["lookaheads"] == h.shape[0] * (L - 1)
    assert ss["offered"] > 0 and ss["words"] > 0 and ss["chunks"] >= ss["words"]
    assert ss["in_time"] > 0, ss
    # a layer only sees streamed jobs whose last chunk was sent (the rest
    # were given back when it entered)
    assert ss["in_time"] + ss["late"] <= ss["words"], ss
    print(f"hits {s['hits']} (without streaming {hits_plain}), stream counters {ss}")
    st.step()
    _check_consistent(st, host)
    st.close()


def test_stream_without_pause_drops_late_and_stays_consistent(weights):
    """No time between layers: most streamed jobs miss their layer; the
    planner drops them (late, or their layer read its table first), their
    slots go back to the pool, and tables stay consistent."""
    _needs_gpu()
    L, host, _ = weights
    h = ar1_states(16, H, seed=6)
    plain = _make(weights, admit="window")
    ref = _run(plain, h)
    plain.close()
    st = _make(weights, admit="window", stream=True, stream_per_layer=4, stream_reserve=2,
               stream_gbps=20.0)
    got = _run(st, h)
    for (y0, i0, _), (y1, i1, _) in zip(ref, got):
        assert np.array_equal(i0, i1)
        assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32))
    ss = st.stream_stats()
    assert ss["lookaheads"] > 0 and ss["offered"] > 0
    _check_consistent(st, host)
    st.close()


def test_stream_prior_sees_published_residency(weights, oracle_lib):
    """Cache prior delta = 0.01 with streaming: at every layer the ids and
    weights equal the oracle router's with the prior on the experts published
    at the last step; a table word a streamed copy wrote within the token
    does not move the router (the reference's prior tensor moves only at
    publication)."""
    _needs_gpu()
    L, host, routers = weights
    Ws = [r.cpu().numpy() for r in routers]
    st = _make(weights, cache_prior=0.01, admit="window", stream=True, stream_per_layer=4,
               stream_reserve=3)
    pub = {}
    mismatched_tables = [0]

    def before_token(t):
        for il in range(L):
            se = st.tables(il)["slot_expert"]
            pub[il] = np.zeros(E, np.float32)
            pub[il][se[se >= 0]] = np.float32(0.01)

    def check(t, il, x, y, ids, w):
        rid, rw, _, _ = oracle_lib.router(Ws[il], x.cpu().numpy()[0], K, pub[il])
        assert np.array_equal(ids.cpu().numpy()[0], rid), f"token {t} layer {il}"
        assert np.array_equal(w.cpu().numpy()[0].view(np.uint32), rw.view(np.uint32)), f"token {t} layer {il}"
        es = st.tables(il)["expert_slot"]
        mismatched_tables[0] += int(((es >= 0) != (pub[il] > 0)).any())

    import time
    h = ar1_states(20, H, seed=8)
    for t in range(h.shape[0]):
        before_token(t)
        x = torch.from_numpy(h[t:t + 1]).cuda()
        for il in range(L):
            y, ids, w = st.layer_forward(il, x)
            check(t, il, x, y, ids, w)
            x = _next_input(x, y)
            torch.cuda.synchronize()
            time.sleep(0.0005)
        st.step()
    ss = st.stream_stats()
    assert ss["words"] > 0, ss
    # the table did move within tokens (streamed words), the router did not
    assert mismatched_tables[0] > 0
    st.step()
    _check_consistent(st, host)
    st.close()


def test_stream_config_rules():
    """moe_create refuses streaming without early issue and out-of-range
    streaming switches."""
    _needs_gpu()
    from moe_prefetch_b200 import MoeCacheConfig, MoeError, MoeStack
    with pytest.raises(MoeError):
        MoeStack(n_layers=1, cache=MoeCacheConfig(n_slots=16, stream=True))
    with pytest.raises(MoeError):
        MoeStack(n_layers=1, cache=MoeCacheConfig(n_slots=16, early_issue=True, stream=True,
                                                  stream_per_layer=17))
    with pytest.raises(MoeError):
        MoeStack(n_layers=1, cache=MoeCacheConfig(n_slots=16, early_issue=True, stream=True,
                                                  stream_topk=17))
