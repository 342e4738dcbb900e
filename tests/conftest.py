import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle.oracle import reference_dir  # noqa: E402

REFERENCE = reference_dir()

# Output tolerances of north_star, against the fp32-accumulated oracle
REL_L2_TOL = 1e-3
MAX_ABS_TOL = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_same_bits(a, b, what):
    """The GEMV paths and the oracle's kernel-order rows (oracle
    or_dot_*_f32, or_combine_f32) round every float step alike: outputs are
    equal bit for bit, not only within the tolerance."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    diff = int((a.view(np.uint32) != b.view(np.uint32)).sum())
    assert diff == 0, f"{what}: {diff} of {a.size} values differ in their bits"


def rms_norm(h, eps=0.0):
    h = np.asarray(h, np.float32)
    return (h / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)).astype(np.float32)


def decode_partition(n_embd, grid):
    """Residual-row ranges [h0, h1) of the persistent decode kernel's CTAs."""
    h0 = np.array([c * n_embd // grid for c in range(grid)], np.int32)
    h1 = np.array([(c + 1) * n_embd // grid for c in range(grid)], np.int32)
    return h0, h1


def with_shared(ids, w, gate, up, down, shared):
    """The expert arrays and pairs with an always-on shared expert appended as
    expert E (weight 1, after the routed ones); unchanged when shared is None."""
    if shared is None:
        return ids, w, gate, up, down
    E = gate.shape[0]
    ids = np.concatenate([ids, np.full(ids.shape[:-1] + (1,), E, np.int32)], axis=-1)
    w = np.concatenate([w, np.ones(w.shape[:-1] + (1,), np.float32)], axis=-1)
    gate, up, down = (np.concatenate([a, np.asarray(b).reshape(1, -1)]) for a, b in zip((gate, up, down), shared))
    return ids, w, gate, up, down


def check_decode_layer(oracle_lib, h_tok, dumps, t, L, W, gate, up, down, grid, n_ff=768,
                       down_type=14, prior=None, shared=None):
    """One (token, layer) of a decode against the oracle: the residual before
    the layer is h + y_0 + ... + y_{L-1} in fp32 (the kernel's order); the
    fused router must give the same ids, weights and normalised x bit for bit;
    the layer output must be within the output tolerance and equal to the
    oracle's kernel-order rows bit for bit.  `shared`: the layer's shared
    expert (gate, up, down bytes) or None."""
    r = np.asarray(h_tok, np.float32).copy()
    ys = dumps["y"]
    for Lp in range(L):
        r = (r + ys[t, Lp]).astype(np.float32)
    h0, h1 = decode_partition(r.size, grid)
    k = dumps["ids"].shape[-1]
    rid, rw, rx, _ = oracle_lib.router_fused(np.ascontiguousarray(W.T), r, k, h0, h1, 1e-6, prior)
    assert np.array_equal(dumps["ids"][t, L], rid), f"ids (t={t}, L={L})"
    assert np.array_equal(dumps["w"][t, L].view(np.uint32), rw.view(np.uint32)), f"w (t={t}, L={L})"
    assert np.array_equal(dumps["x"][t, L].view(np.uint32), rx.view(np.uint32)), f"x (t={t}, L={L})"
    xi, xw, xg, xu, xd = with_shared(rid[None], rw[None], gate, up, down, shared)
    ry = oracle_lib.moe_experts(rx[None], xi, xw, xg, xu, xd, down_type, n_ff)[0]
    assert rel_l2(ys[t, L], ry) <= REL_L2_TOL, (t, L, rel_l2(ys[t, L], ry))
    assert np.abs(ys[t, L] - ry).max() <= MAX_ABS_TOL
    assert_same_bits(ys[t, L], ry, f"layer output (t={t}, L={L})")


def ar1_states(n_tok, n_embd, rho=0.9, seed=12345):
    """AR(1) hidden states h_t = rho h_{t-1} + sqrt(1-rho^2) eps_t, RMS-normed."""
    rng = np.random.default_rng(seed)
    h = np.empty((n_tok, n_embd), np.float32)
    prev = rng.standard_normal(n_embd)
    for t in range(n_tok):
        prev = rho * prev + np.sqrt(1 - rho * rho) * rng.standard_normal(n_embd)
        h[t] = prev
    return rms_norm(h)


def toy_moep(n_layers, n_expert, layers, seed, blocks=(1, 2, 3, 4), prior=0.25):
    """A seeded MOEP v3 model (moe_prefetch_b200.predictor.MoePredictor) with
    the given layers and feature blocks (1 prev, 2 cur, 3 below, 4
    self_prev), N(0, 1) weights and biases: a stand-in for a trained
    evictor or predictor."""
    from moe_prefetch_b200.predictor import MoePredictor
    rng = np.random.default_rng(seed)
    p = MoePredictor()
    p.n_expert, p.n_layers, p.top_k = n_expert, n_layers, 8
    for i, kind in enumerate(blocks):
        p.off[kind] = i * n_expert
    p.feat_dim = len(blocks) * n_expert
    p.layer_of = np.asarray(layers, np.int32)
    p.index_of = np.full(n_layers, -1, np.int32)
    for i, il in enumerate(layers):
        p.index_of[il] = i
    p.prior = np.full(len(layers), prior, np.float32)
    p.bias = rng.standard_normal((len(layers), n_expert)).astype(np.float32)
    p.w = rng.standard_normal((len(layers), p.feat_dim, n_expert)).astype(np.float32)
    return p
