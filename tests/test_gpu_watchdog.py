"""The decode kernel's watchdog: a device wait that runs out is reported as
MOE_ERR_TIMEOUT once, and the context stays usable.

The reference's counterpart is the sidecar deadline: when the host side stops
answering, llama_context::decode returns -3 and the next decode proceeds
(patches/0009:652-655; cpp/test-moe-sidecar.cpp's dead-host case).  Here the
wait that runs out is one rank's activation signal, made unreachable through
the test-only `starve` field of moe_decode_dbg (its first wait targets one
signal more than its producers give).  Nothing faults: every CTA sees the
abort flag, waits (bounded) for its own copies and returns.
"""
import numpy as np
import pytest

from conftest import ar1_states

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H = 2048


@pytest.fixture(scope="module")
def stack():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    st = MoeStack(n_layers=3)
    st.synth_resident(seed=5, keep_router=True)
    yield st
    st.set_wait_limit(0)
    st.close()


def test_starved_wait_reports_timeout_then_recovers(stack):
    from moe_prefetch_b200._lib import MoeError
    st = stack
    h = ar1_states(3, H, seed=31)
    hp = torch.from_numpy(h).pin_memory()
    ref = torch.empty_like(hp).pin_memory()
    st.decode_host(hp, ref)                      # default 2 s limit, clean run
    st.set_wait_limit(2_000_000)                 # 2 ms: a normal 3-token call takes ~0.2 ms
    for rank in (1, 8):                          # the first and the last routed rank
        with pytest.raises(MoeError) as ei:
            st.decode(torch.from_numpy(h).cuda(), starve=rank)
            st.sync()
        assert ei.value.code == -5, str(ei.value)   # MOE_ERR_TIMEOUT
        st.sync()                                    # reported once: clean now
        out = torch.empty_like(hp).pin_memory()
        st.decode_host(hp, out)                      # the next call is correct
        assert torch.equal(out, ref)
    # unsynchronised: the flag surfaces at the next moe_decode_host, once,
    # and the call after that is clean
    st.decode(torch.from_numpy(h).cuda(), starve=4)
    out = torch.empty_like(hp).pin_memory()
    with pytest.raises(MoeError) as ei:
        st.decode_host(hp, out)
    assert ei.value.code == -5
    st.decode_host(hp, out)
    assert torch.equal(out, ref)
    st.set_wait_limit(0)
    st.decode_host(hp, out)
    assert torch.equal(out, ref)


def test_starve_out_of_range_is_an_argument_error(stack):
    from moe_prefetch_b200._lib import MoeError
    h = torch.from_numpy(ar1_states(1, H, seed=2)).cuda()
    with pytest.raises(MoeError) as ei:
        stack.decode(h, starve=99)
    assert ei.value.code == -1
    assert np.isfinite(stack.decode(h).cpu().numpy()).all()
    stack.sync()
