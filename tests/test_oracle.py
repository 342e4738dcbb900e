"""The CPU oracle pinned against its golden sources: ggml block decode against
gguf-py 0.19.0 (fixture + live when installed), fp16 conversion against
numpy, exp against libm, the router's selection rules, the Q8_1 / Q8_K
activation paths against a plain fp32 reference."""
import math
import os

import numpy as np
import pytest

from conftest import rel_l2, rms_norm

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def test_decode_matches_gguf_fixture(oracle_lib):
    d = np.load(os.path.join(GOLD, "q4k_q6k_gguf.npz"))
    for name, qt in (("q4k", 12), ("q6k", 14)):
        x = d[f"{name}_x"]
        blocks = d[f"{name}_blocks"]
        assert np.array_equal(oracle_lib.quantize(x, qt), blocks), "quantiser drifted"
        got = oracle_lib.dequantize(blocks, qt, x.size)
        assert np.array_equal(got, d[f"{name}_deq"]), f"{name} decode differs from gguf-py"


def test_decode_matches_gguf_live(oracle_lib):
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T
    from gguf import quants
    rng = np.random.default_rng(1)
    for qt, gt, scale in ((12, T.Q4_K, 0.02), (14, T.Q6_K, 0.02), (12, T.Q4_K, 3.0),
                          (14, T.Q6_K, 5.0)):
        x = (rng.standard_normal(256 * 64) * scale).astype(np.float32)
        y = oracle_lib.quantize(x, qt)
        assert np.array_equal(oracle_lib.dequantize(y, qt, x.size),
                              quants.dequantize(y, gt).ravel().astype(np.float32))
    del gguf


def test_quantiser_error_bounds(oracle_lib):
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(256 * 256) * 0.02).astype(np.float32)
    e4 = rel_l2(oracle_lib.dequantize(oracle_lib.quantize(x, 12), 12, x.size), x)
    e6 = rel_l2(oracle_lib.dequantize(oracle_lib.quantize(x, 14), 14, x.size), x)
    assert e4 < 0.1 and e6 < 0.03, (e4, e6)


def test_f16_round_to_nearest_even(oracle_lib):
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                           for s in (1e-6, 1e-3, 1.0, 1e3, 6e4)] +
                          [np.array([0.0, -0.0, 65504.0, 70000.0, 1e-8, 5.96e-8], np.float32)])
    for v in vals:
        with np.errstate(over="ignore"):
            ref = np.float32(v).astype(np.float16).view(np.uint16)
        assert oracle_lib.f32_to_f16_bits(v) == ref


def test_expf_within_one_ulp(oracle_lib):
    for x in np.linspace(-79.0, 10.0, 4001).astype(np.float32):
        got = np.float32(oracle_lib.expf(x))
        ref = np.float32(math.exp(float(x)))
        ulp = np.spacing(ref)
        assert abs(float(got) - math.exp(float(x))) <= 1.0 * float(ulp), x
    assert oracle_lib.expf(-100.0) == 0.0


def test_router_selection_rules(oracle_lib):
    rng = np.random.default_rng(4)
    E, H = 128, 2048
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rms_norm(rng.standard_normal(H))
    ids, w, p, lg = oracle_lib.router(W, x, 8)
    assert len(set(ids)) == 8
    assert np.all(np.diff(p[ids]) <= 0), "ids must be in descending selection order"
    assert abs(float(w.sum()) - 1.0) < 1e-6
    assert np.allclose(p, np.exp(lg - lg.max()) / np.exp(lg - lg.max()).sum(), rtol=1e-5)
    assert np.allclose(lg, W.astype(np.float64) @ x, atol=1e-5)
    # ties: zero input -> equal logits -> lowest ids
    ids0, w0, _, _ = oracle_lib.router(W, np.zeros(H, np.float32), 8)
    assert list(ids0) == list(range(8)) and np.allclose(w0, 0.125)
    # prior: a resident expert ranked within delta wins, weights stay unbiased
    prior = np.zeros(E, np.float32)
    cand = int(np.argsort(-p)[8])                   # the 9th best
    prior[cand] = np.float32(p[ids[7]] - p[cand] + 1e-4)
    ids2, w2, p2, _ = oracle_lib.router(W, x, 8, prior)
    assert cand in ids2
    assert np.array_equal(p2, p)
    assert np.allclose(w2, p[ids2] / p[ids2].sum(), rtol=1e-6)


def test_q8_1_quantisation(oracle_lib):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(2048).astype(np.float32)
    q, d, s = oracle_lib.quantize_q8_1(x)
    xb = x.reshape(-1, 32)
    assert np.allclose(d, np.abs(xb).max(1) / 127, rtol=1e-7)
    assert np.abs(q).max() <= 127
    assert np.allclose(s, d * q.reshape(-1, 32).sum(1), rtol=1e-6)
    rec = (q.reshape(-1, 32) * d[:, None]).ravel()
    assert np.abs(rec - x).max() <= d.max() / 2 + 1e-6


def test_expert_row_paths_agree(oracle_lib):
    """The Q8_1 path (the parity oracle) and the Q8_K path (ggml's CPU
    activation format) both approximate the fp32 expert; the gap between them
    is the activation quantisation (~1e-2), which is why the parity bar uses
    the same activation format as the kernel."""
    rng = np.random.default_rng(6)
    H, I = 2048, 256
    g = oracle_lib.quantize((rng.standard_normal((I, H)) * 0.02).astype(np.float32), 12)
    u = oracle_lib.quantize((rng.standard_normal((I, H)) * 0.02).astype(np.float32), 12)
    dn = oracle_lib.quantize((rng.standard_normal((H, I)) * 0.02).astype(np.float32), 14)
    x = rms_norm(rng.standard_normal(H))
    y1, _ = oracle_lib.expert_row(g, u, dn, 14, H, I, x)
    y2, _ = oracle_lib.expert_row(g, u, dn, 14, H, I, x, q8K=True)
    # fp32 reference on the dequantised weights
    G = oracle_lib.dequantize(g, 12, I * H).reshape(I, H).astype(np.float64)
    U = oracle_lib.dequantize(u, 12, I * H).reshape(I, H).astype(np.float64)
    D = oracle_lib.dequantize(dn, 14, H * I).reshape(H, I).astype(np.float64)
    gg, uu = G @ x, U @ x
    act = gg / (1 + np.exp(-gg)) * uu
    yr = D @ act
    assert rel_l2(y1, yr) < 0.03 and rel_l2(y2, yr) < 0.03
    assert rel_l2(y1, y2) < 0.05


def test_cpu_fast_path_matches_q8K_oracle(oracle_lib):
    rng = np.random.default_rng(7)
    H, I, E, K = 2048, 256, 32, 8
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    g = oracle_lib.quantize((rng.standard_normal((E * I, H)) * 0.02).astype(np.float32), 12).reshape(E, -1)
    u = oracle_lib.quantize((rng.standard_normal((E * I, H)) * 0.02).astype(np.float32), 12).reshape(E, -1)
    d = oracle_lib.quantize((rng.standard_normal((E * H, I)) * 0.02).astype(np.float32), 14).reshape(E, -1)
    x = rms_norm(rng.standard_normal(H))
    ids, w, y = oracle_lib.moe_layer_cpu_fast(x, W, g, u, d, 14, I, K, n_threads=4)
    rids, rw, ry = oracle_lib.moe_layer(x[None], W, g, u, d, 14, I, K, path="q8K")
    assert np.array_equal(ids, rids[0]) and np.array_equal(w, rw[0])
    assert rel_l2(y, ry[0]) < 1e-5


@pytest.mark.parametrize("qtype,n", [(12, 2048), (12, 768), (14, 768), (14, 512), (12, 4096)])
def test_kernel_order_dots_match_double(oracle_lib, qtype, n):
    """The kernel-order fp32 dots (unit partials, lane butterfly / row-group
    tree) are the double-accumulated dots up to fp32 rounding, relative to
    the sum of the products' magnitudes."""
    rng = np.random.default_rng(11 + n)
    rows = oracle_lib.quantize((rng.standard_normal((64, n)) * 0.02).astype(np.float32), qtype)
    q, d, s = oracle_lib.quantize_q8_1(rms_norm(rng.standard_normal(n)))
    err = 0.0
    for r in rows:
        a = oracle_lib.dot_q8_1(r, qtype, q, d, s)
        b = oracle_lib.dot_q8_1(r, qtype, q, d, s, order="kernel")
        scale = np.abs(oracle_lib.dequantize(r, qtype, n)).sum() * np.abs(q * np.repeat(d, 32)).max()
        err = max(err, abs(a - b) / scale)
    assert err < 1e-6
