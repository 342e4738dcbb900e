"""Expert parallelism on GPUs, through the C ABI.

- World size 1 (one GPU, no process group): the three EP device steps must
  reproduce moe_layer_forward_path:
  - the GEMV path bit for bit;
  - the GEMM path bit for bit as well: the expert tiles hold the same pairs
    in the same order.
- World size 2 (two GPUs): tests/ep_worker.py under torch.distributed.run,
  with the NCCL exchange and with the peer-memory mailboxes (eager and
  captured in a CUDA graph), against a single-GPU stack with the same
  weights; skipped on one GPU.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import rms_norm

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H = 2048
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module", params=[(128, 768, 0), (256, 512, 1)], ids=["c1", "c4shared"])
def stacks(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_prefetch_b200 import MoeStack
    from moe_prefetch_b200.ep import ExpertParallelStack
    E, I, n_shared = request.param
    ep = ExpertParallelStack(1, n_expert=E, n_ff=I, n_shared=n_shared)
    ep.synth(seed=29)
    ref = MoeStack(n_layers=1, n_expert=E, n_ff=I, n_shared=n_shared)
    ref.synth_resident(seed=29)
    yield ep, ref
    ep.close()
    ref.close()


@pytest.mark.parametrize("path,n_tok", [("gemv", 5), ("gemv", 40), ("gemm", 40), ("gemm", 130)])
def test_ep_world1_equals_layer(stacks, path, n_tok):
    ep, ref = stacks
    X = torch.from_numpy(rms_norm(np.random.default_rng(n_tok).standard_normal((n_tok, H)))).cuda()
    out, ids, w = ep.layer_forward(0, X, path)
    y, rids, rw = ref.layer_forward_path(0, X, path)
    torch.cuda.synchronize()
    assert torch.equal(ids, rids) and torch.equal(w.view(torch.int32), rw.view(torch.int32))
    assert torch.equal(out.view(torch.int32), y.view(torch.int32))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "ep_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "EP_OK" in r.stdout, r.stdout[-3000:]
