"""The tensor-core grouped GEMM path (tcgen05) against the oracle, through the C ABI.

moe_layer_forward_path(..., MOE_PATH_GEMM) groups the routed pairs by expert,
dequantises Q4_K/Q6_K rows to fp16 in shared memory and runs tcgen05.mma with
fp32 accumulators in TMEM.  Bars:
- ids and routing weights bit-exact: the same router as every path;
- outputs within relative L2 <= 1e-3 and max-abs <= 1e-2 of the oracle's
  fp32 reference: exact dequantised weights times unquantised activations,
  fp64 accumulation.
"""
import numpy as np
import pytest

from conftest import MAX_ABS_TOL, REL_L2_TOL, rel_l2, rms_norm

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8
Q6K = 14


@pytest.fixture(scope="module")
def layer(oracle_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=1)
    st.synth_resident(seed=19, keep_router=True)
    g, u, d = st.slot_views(0)
    W = st.routers[0].cpu().numpy()
    gate, up, down = (v[:E].cpu().numpy() for v in (g, u, d))
    yield st, W, gate, up, down
    st.close()


def _check(oracle_lib, layer, X, path="gemm"):
    st, W, gate, up, down = layer
    y, ids, w = st.layer_forward_path(0, torch.from_numpy(X).cuda(), path)
    st.sync()
    y, ids, w = y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()
    rids, rw, _ = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K)
    assert np.array_equal(ids, rids)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    ry = oracle_lib.moe_experts(X, ids, w, gate, up, down, Q6K, I, path="f32")
    assert np.isfinite(y).all()
    print(f"n_tok {X.shape[0]}: rel L2 {rel_l2(y, ry):.3e}, max abs {np.abs(y - ry).max():.3e}")
    assert rel_l2(y, ry) <= REL_L2_TOL, rel_l2(y, ry)
    assert np.abs(y - ry).max() <= MAX_ABS_TOL, np.abs(y - ry).max()
    return y, ry


@pytest.mark.parametrize("n_tok", [2, 16, 64, 200, 512])
def test_gemm_matches_f32_reference(oracle_lib, layer, n_tok):
    """Up to the 512-token prefill chunk of the benchmarks (4096 pairs, about
    32 per expert: tiles of every size)."""
    X = rms_norm(np.random.default_rng(900 + n_tok).standard_normal((n_tok, H)))
    _check(oracle_lib, layer, X)


def test_gemm_expert_spanning_two_token_tiles(oracle_lib, layer):
    """96 identical tokens: each of the 8 routed experts gets 96 pairs, i.e. a
    full 64-pair tile and a 32-pair tile; 120 experts get none."""
    x1 = rms_norm(np.random.default_rng(41).standard_normal((1, H)))
    X = np.repeat(x1, 96, axis=0)
    y, _ = _check(oracle_lib, layer, X)
    assert (y == y[:1]).all()


def test_gemm_two_calls_in_a_row_reuse_scratch(oracle_lib, layer):
    """A large batch then a small one: stale tiles of the first call must not
    leak into the second."""
    rng = np.random.default_rng(5)
    _check(oracle_lib, layer, rms_norm(rng.standard_normal((150, H))))
    _check(oracle_lib, layer, rms_norm(rng.standard_normal((3, H))))


def test_auto_path_choice(oracle_lib, layer):
    """auto takes the GEMM from 4 pairs per expert on (n_tok * 8 >= 512) and
    the Q8_1 GEMV below: the small batch is bit-identical to the GEMV path."""
    st = layer[0]
    X = torch.from_numpy(rms_norm(np.random.default_rng(6).standard_normal((8, H)))).cuda()
    ya, _, _ = st.layer_forward_path(0, X, "auto")
    yv, _, _ = st.layer_forward_path(0, X, "gemv")
    st.sync()
    assert torch.equal(ya.view(torch.int32), yv.view(torch.int32))
    Xb = rms_norm(np.random.default_rng(7).standard_normal((64, H)))
    yb, _, _ = st.layer_forward_path(0, torch.from_numpy(Xb).cuda(), "auto")
    yg, _, _ = st.layer_forward_path(0, torch.from_numpy(Xb).cuda(), "gemm")
    st.sync()
    assert torch.equal(yb.view(torch.int32), yg.view(torch.int32))
