"""Config-4 shapes on the GPU: 256 routed experts, intermediate 512, and one
always-on shared expert per layer (weight 1, after the k routed experts).

Every path must match the oracle, with the shared expert appended as expert
256 of the weight arrays and as a ninth pair (256, 1.0) per token:
- per-pair GEMV (one token) and grouped GEMV (a batch): Q8_1 arithmetic;
- the tcgen05 GEMM: against the f32 reference;
- the persistent decode kernel: fused router bit for bit, layer outputs within
  tolerance.
Ids and weights are the k routed ones and must be bit-exact.
"""
import numpy as np
import pytest

from conftest import (MAX_ABS_TOL, REL_L2_TOL, ar1_states, check_decode_layer, rel_l2, rms_norm,
                      with_shared)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 512, 256, 8
Q6K = 14


@pytest.fixture(scope="module")
def c4(oracle_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=2, n_expert=E, n_ff=I, n_shared=1)
    st.synth_resident(seed=61, keep_router=True)
    layers = []
    for il in range(2):
        g, u, d = st.slot_views(il)
        W = st.routers[il].cpu().numpy()
        sh = tuple(v.cpu().numpy() for v in st.shared[il])
        layers.append((W, g[:E].cpu().numpy(), u[:E].cpu().numpy(), d[:E].cpu().numpy(), sh))
    yield st, layers
    st.close()


def _check(oracle_lib, layer, X, y, ids, w, path="q8_1"):
    W, gate, up, down, sh = layer
    rids, rw, _ = oracle_lib.moe_layer(X, W, gate, up, down, Q6K, I, K)
    assert np.array_equal(ids, rids)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    xi, xw, xg, xu, xd = with_shared(rids, rw, gate, up, down, sh)
    ry = oracle_lib.moe_experts(X, xi, xw, xg, xu, xd, Q6K, I, path=path)
    assert rel_l2(y, ry) <= REL_L2_TOL, rel_l2(y, ry)
    assert np.abs(y - ry).max() <= MAX_ABS_TOL


@pytest.mark.parametrize("n_tok", [1, 24])
def test_shared_gemv_paths(oracle_lib, c4, n_tok):
    st, layers = c4
    X = rms_norm(np.random.default_rng(70 + n_tok).standard_normal((n_tok, H)))
    y, ids, w = st.layer_forward(1, torch.from_numpy(X).cuda())
    st.sync()
    _check(oracle_lib, layers[1], X, y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy())


def test_shared_gemm_path(oracle_lib, c4):
    st, layers = c4
    X = rms_norm(np.random.default_rng(80).standard_normal((96, H)))
    y, ids, w = st.layer_forward_path(0, torch.from_numpy(X).cuda(), "gemm")
    st.sync()
    _check(oracle_lib, layers[0], X, y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), path="f32")


@pytest.mark.parametrize("spec", [0, 2])
def test_shared_decode(oracle_lib, c4, spec):
    """spec 2: a wrong prediction in every other (token, layer), so that the
    shared expert's pieces are re-issued too."""
    st, layers = c4
    n_tok = 3
    h = ar1_states(n_tok, H, seed=9)
    out, dm = st.decode(torch.from_numpy(h).cuda(), debug=True, spec=spec)
    st.sync()
    dumps = {k: v.cpu().numpy() for k, v in dm.items()}
    grid = st.decode_info()["grid"]
    for t in range(n_tok):
        for il in range(2):
            W, gate, up, down, sh = layers[il]
            check_decode_layer(oracle_lib, h[t], dumps, t, il, W, gate, up, down, grid, n_ff=I,
                               shared=sh)


def test_shared_must_be_set(c4):
    from moe_prefetch_b200 import MoeStack
    from moe_prefetch_b200._lib import MoeError
    st = MoeStack(n_layers=1, n_expert=E, n_ff=I, n_shared=1)
    try:
        with pytest.raises(MoeError):
            st.layer_forward(0, torch.zeros(1, H, device="cuda"))
    finally:
        st.close()


def test_noalloc_refuses_shared_expert(c4):
    """The allocation-free layer entry point does not run shared experts: a
    context with n_shared = 1 gets MOE_ERR_UNSUPPORTED, and nothing is written."""
    from moe_prefetch_b200._lib import MoeError
    st, _ = c4
    x = torch.from_numpy(rms_norm(np.random.default_rng(3).standard_normal((2, H)))).cuda()
    y = torch.full((2, H), 7.0, device="cuda")
    with pytest.raises(MoeError) as ei:
        st.layer_forward_noalloc(0, x, y)
    assert ei.value.code == -4
    assert torch.all(y == 7.0)
