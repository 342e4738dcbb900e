"""Worker of tests/test_gpu_ep.py: expert parallelism, one rank per GPU.

For two stacks -- config 1's shapes, and config 4's (256 experts, n_ff 512,
one always-on shared expert) -- and both exchanges (NCCL all-to-all, and the
library's peer-memory mailboxes), every rank builds its share of a 2-layer
stack (ExpertParallelStack.synth), runs both layers on its home tokens for
the GEMV and the GEMM paths, and all-gathers the outputs.  With the
mailboxes it also captures the two GEMV layers in a CUDA graph and replays
it twice on new inputs.  Rank 0 then builds the whole stack on its own GPU
with the same seed (MoeStack.synth_resident) and checks:
- the GEMV path bit for bit (the replays too);
- the GEMM path within the layer tolerance.
Prints EP_OK on success; exits non-zero otherwise.  Launched with
torch.distributed.run; MASTER_ADDR 127.0.0.1.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

H, L, SEED, TOK_PER_RANK = 2048, 2, 23, 40


def rms(h):
    return (h / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True))).astype(np.float32)


def main():
    from moe_prefetch_b200 import MoeStack
    from moe_prefetch_b200.ep import ExpertParallelStack
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ok = True
    try:
        for exchange in ("nccl", "peer"):
            for shape in ((128, 768, 0), (256, 512, 1)):
                ok = run_shape(rank, world, shape, exchange, MoeStack, ExpertParallelStack) and ok
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.broadcast(flag, 0)
        ok = bool(flag.item())
    finally:
        dist.destroy_process_group()
    if rank == 0 and ok:
        print("EP_OK")
    return 0 if ok else 1


def gather(out, ids):
    world = dist.get_world_size()
    allo = torch.empty(world, *out.shape, device=out.device)
    alli = torch.empty(world, *ids.shape, dtype=ids.dtype, device=ids.device)
    dist.all_gather_into_tensor(allo, out.contiguous())
    dist.all_gather_into_tensor(alli, ids.contiguous())
    return allo.cpu().numpy(), alli.cpu().numpy()


def run_shape(rank, world, shape, exchange, MoeStack, ExpertParallelStack):
    E, I, n_shared = shape
    ok = True
    ep = ExpertParallelStack(L, n_expert=E, n_ff=I, n_shared=n_shared, exchange=exchange,
                             max_home_tokens=TOK_PER_RANK)
    ep.synth(SEED)
    X = rms(np.random.default_rng(100).standard_normal((world * TOK_PER_RANK, H)))
    mine = torch.from_numpy(X[rank::world].copy()).cuda()
    got = {}
    for path in ("gemv", "gemm"):
        for layer in range(L):
            out, ids, w = ep.layer_forward(layer, mine, path)
            got[(path, layer, 0)] = gather(out, ids)
    Xg = []
    if exchange == "peer":
        # both GEMV layers in one CUDA graph: nothing in them waits for the host
        xin = torch.zeros_like(mine)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                outs = [ep.layer_forward(layer, xin, "gemv") for layer in range(L)]
        torch.cuda.current_stream().wait_stream(s)
        for rep in (1, 2):
            Xr = rms(np.random.default_rng(100 + rep).standard_normal((world * TOK_PER_RANK, H)))
            Xg.append(Xr)
            xin.copy_(torch.from_numpy(Xr[rank::world].copy()).cuda())
            g.replay()
            torch.cuda.synchronize()
            for layer in range(L):
                got[("gemv", layer, rep)] = gather(outs[layer][0], outs[layer][1])
        del g
    torch.cuda.synchronize()
    if rank == 0:
        ref = MoeStack(n_layers=L, n_expert=E, n_ff=I, n_shared=n_shared)
        ref.synth_resident(seed=SEED)
        for (path, layer, rep), (allo, alli) in got.items():
            Xin = X if rep == 0 else Xg[rep - 1]
            y, ids, _ = ref.layer_forward_path(layer, torch.from_numpy(Xin).cuda(), path)
            y, ids = y.cpu().numpy(), ids.cpu().numpy()
            for r in range(world):
                yr, ir = y[r::world], ids[r::world]
                if not np.array_equal(alli[r], ir):
                    print(f"ids differ: {exchange} path {path} layer {layer} rep {rep} rank {r}")
                    ok = False
                if path == "gemv":
                    same = np.array_equal(allo[r].view(np.uint32), yr.view(np.uint32))
                else:
                    rel = np.linalg.norm(allo[r] - yr) / np.linalg.norm(yr)
                    same = rel <= 1e-3 and np.abs(allo[r] - yr).max() <= 1e-2
                if not same:
                    print(f"outputs differ: {exchange} shape {shape} path {path} layer {layer} rep {rep} rank {r}")
                    ok = False
        ref.close()
    ep.close()
    return ok


if __name__ == "__main__":
    sys.exit(main())
