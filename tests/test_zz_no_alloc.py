"""moe_layer_forward_noalloc against moe_layer_forward, through the C ABI.

The no-allocation variant keeps its scratch in a static per-device array
instead of buffers grown with cudaMalloc.  Its results must match the
allocating entry point's on the same inputs: ids and routing weights
bit-exact, outputs within relative L2 <= 1e-3 and max-abs <= 1e-2.  The
checks make two calls in a row, with different inputs and batch sizes, so
that stale scratch from the first call cannot leak into the second.  The file
is named to be collected last.  It passes on its own, where its first call
sets the scratch up, and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import MAX_ABS_TOL, REL_L2_TOL, rel_l2, rms_norm

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8
SCRATCH_BYTES = 4 << 20          # MOE_NOALLOC_SCRATCH_BYTES
MAX_TOK = 170                    # largest n_tok that fits for n_used 8, n_ff 768
MOE_ERR_ARG = -1
MOE_ERR_UNSUPPORTED = -4


def _need(n_tok):
    r256 = lambda b: (b + 255) // 256 * 256
    return 2 * r256(4 * n_tok * K) + 4 * n_tok * K * I


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _s():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def stack():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=2)
    st.synth_resident(seed=31, keep_router=True)
    assert st.n_used == K and st.n_ff == I and st.n_embd == H
    yield st
    st.close()


def _noalloc(st, layer, x, with_sel=True):
    """One call of the C entry point; returns (y, ids, w) (ids/w None when the
    selection stays in the scratch)."""
    n_tok = x.shape[0]
    y = torch.full_like(x, float("nan"))
    ids = torch.full((n_tok, K), -7, dtype=torch.int32, device=x.device) if with_sel else None
    w = torch.full((n_tok, K), float("nan"), device=x.device) if with_sel else None
    rc = st.lib.moe_layer_forward_noalloc(st.ctx, layer, _p(x), _p(y), n_tok, _p(ids), _p(w), _s())
    assert rc == 0, st.lib.moe_last_error(st.ctx)
    return y, ids, w


def _compare(y, ids, w, ry, rids, rw):
    y, ry = y.cpu().numpy(), ry.cpu().numpy()
    assert np.isfinite(y).all()
    if ids is not None:
        assert np.array_equal(ids.cpu().numpy(), rids.cpu().numpy())
        assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.cpu().numpy().view(np.uint32))
    assert rel_l2(y, ry) <= REL_L2_TOL, rel_l2(y, ry)
    assert np.abs(y - ry).max() <= MAX_ABS_TOL


def test_scratch_limit_formula():
    assert _need(MAX_TOK) <= SCRATCH_BYTES < _need(MAX_TOK + 1)


@pytest.mark.parametrize("with_sel", [True, False])
def test_noalloc_matches_layer_forward_two_calls(stack, with_sel):
    st = stack
    rng = np.random.default_rng(8 if with_sel else 9)
    X1 = torch.from_numpy(rms_norm(rng.standard_normal((48, H)))).cuda()
    X2 = torch.from_numpy(rms_norm(rng.standard_normal((5, H)))).cuda()
    for layer, x in ((0, X1), (1, X2)):           # two calls in a row
        y, ids, w = _noalloc(st, layer, x, with_sel)
        ry, rids, rw = st.layer_forward(layer, x)
        st.sync()
        _compare(y, ids, w, ry, rids, rw)


def test_noalloc_batch1_then_max_batch(stack):
    st = stack
    rng = np.random.default_rng(10)
    X1 = torch.from_numpy(rms_norm(rng.standard_normal((1, H)))).cuda()
    X2 = torch.from_numpy(rms_norm(rng.standard_normal((MAX_TOK, H)))).cuda()
    outs = [_noalloc(st, 0, X1), _noalloc(st, 0, X2)]    # back to back, one stream
    refs = [st.layer_forward(0, X1), st.layer_forward(0, X2)]
    st.sync()
    for (y, ids, w), (ry, rids, rw) in zip(outs, refs):
        _compare(y, ids, w, ry, rids, rw)


def test_noalloc_rejects_batches_beyond_the_scratch(stack):
    st = stack
    x = torch.zeros(MAX_TOK + 1, H, device="cuda")
    y = torch.zeros_like(x)
    rc = st.lib.moe_layer_forward_noalloc(st.ctx, 0, _p(x), _p(y), MAX_TOK + 1, None, None, _s())
    assert rc == MOE_ERR_ARG
    msg = st.lib.moe_last_error(st.ctx).decode()
    assert "at most 170 tokens" in msg, msg
    assert torch.count_nonzero(y).item() == 0      # nothing was launched
    from moe_prefetch_b200._lib import MoeError
    with pytest.raises(MoeError):
        st.layer_forward_noalloc(0, x, y)


def test_noalloc_refuses_shared_expert_contexts(stack):
    """A context with an always-on shared expert is refused before anything
    is launched (the allocating entry point serves it)."""
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=1, n_expert=256, n_ff=512, n_shared=1)
    try:
        x = torch.zeros(2, H, device="cuda")
        y = torch.zeros_like(x)
        rc = st.lib.moe_layer_forward_noalloc(st.ctx, 0, _p(x), _p(y), 2, None, None, _s())
        assert rc == MOE_ERR_UNSUPPORTED
        assert "shared expert" in st.lib.moe_last_error(st.ctx).decode()
        assert torch.count_nonzero(y).item() == 0
    finally:
        st.close()
