"""Expert-parallel orchestration at world size 2 on the CPU (gloo).

ep_layer_forward exchanges counts, expert ids and token rows all-to-all, lets
each rank run its own experts on what it received, exchanges the rows back and
combines them in rank order.  Here the three device steps are played by the
oracle: routing, the expert rows (Q8_1 arithmetic, k = 1, unweighted) and the
combine (fp64, rank order, as the oracle's own layer).  The EP result must
therefore equal the single-process oracle layer bit for bit.  The checks
include a rank that owns no routed expert (experts 16..31) and receives no rows.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

H, I, E, K = 2048, 768, 32, 4


def _weights(skew):
    import oracle
    rng = np.random.default_rng(3)
    gate = oracle.quantize((rng.standard_normal((E * I, H)) * 0.02).astype(np.float32), 12).reshape(E, -1)
    up = oracle.quantize((rng.standard_normal((E * I, H)) * 0.02).astype(np.float32), 12).reshape(E, -1)
    down = oracle.quantize((rng.standard_normal((E * H, I)) * 0.02).astype(np.float32), 14).reshape(E, -1)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    X = rng.standard_normal((12, H)).astype(np.float32)
    if skew:   # rank 1's experts never win: positive logits only for 0..15
        W = np.abs(W)
        W[E // 2:] = 0.0
        X = np.abs(X)
    X = (X / np.sqrt((X.astype(np.float64) ** 2).mean(-1, keepdims=True))).astype(np.float32)
    return W, gate, up, down, X


class OracleOps:
    """route_pack / experts_rows / combine of ep_layer_forward, on the oracle."""

    def __init__(self, W, gate, up, down, rank, world):
        self.W, self.gate, self.up, self.down = W, gate, up, down
        self.per = E // world
        self.e0 = rank * self.per

    n_used = K

    def route_pack(self, layer, x, world, capacity=0):
        import oracle
        xn = x.numpy()
        n_tok = xn.shape[0]
        ids = np.empty((n_tok, K), np.int32)
        w = np.empty((n_tok, K), np.float32)
        for t in range(n_tok):
            ids[t], w[t], _, _ = oracle.router(self.W, xn[t], K)
        flat = ids.ravel()
        dest = flat // self.per
        order = np.argsort(dest, kind="stable")          # rank order, pair order within
        send_count = np.bincount(dest, minlength=world).astype(np.int32)
        if capacity == 0:
            slot = np.arange(flat.size)
            send_ids, send_x = flat[order].copy(), xn[order // K].copy()
        else:                                            # rank d's block at d * capacity
            start = np.concatenate([[0], np.cumsum(send_count)[:-1]])
            q = np.arange(flat.size)
            slot = dest[order] * capacity + (q - start[dest[order]])
            send_ids = np.full(world * capacity, -1, np.int32)
            send_x = np.zeros((world * capacity, xn.shape[1]), np.float32)
            send_ids[slot] = flat[order]
            send_x[slot] = xn[order // K]
        pos = np.empty(flat.size, np.int32)
        pos[order] = slot
        return (torch.from_numpy(ids), torch.from_numpy(w), torch.from_numpy(send_count),
                torch.from_numpy(pos), torch.from_numpy(send_ids), torch.from_numpy(send_x))

    def experts_rows(self, layer, x_rows, ids, path):
        import oracle
        n = x_rows.shape[0]
        if n == 0:
            return torch.empty(0, H)
        ids = ids.numpy()
        live = ids >= 0                                  # -1: an empty capacity slot
        assert ((ids[live] >= self.e0) & (ids[live] < self.e0 + self.per)).all(), "a row reached a non-owner"
        y = np.zeros((n, H), np.float32)
        if live.any():
            y[live] = oracle.moe_experts(x_rows.numpy()[live], ids[live][:, None],
                                         np.ones((int(live.sum()), 1), np.float32), self.gate, self.up,
                                         self.down, 14, I, n_threads=2)
        return torch.from_numpy(y)

    def combine(self, back, pos, w, n_tok, add_rows=None):
        import oracle
        assert add_rows is None
        rows = back.numpy()[pos.numpy().reshape(n_tok, K)]     # [n_tok, K, H]
        return torch.from_numpy(oracle.combine_rows(w.numpy(), rows))   # the kernels' order


def _worker(rank, world, port, skew, capacity, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from moe_prefetch_b200.ep import ep_layer_forward
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, gate, up, down, X = _weights(skew)
        mine = X[rank::world]                                 # this rank's home tokens
        ops = OracleOps(W, gate, up, down, rank, world)
        out, ids, w = ep_layer_forward(ops, 0, torch.from_numpy(mine), capacity=capacity)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("skew", [False, True])
@pytest.mark.parametrize("capacity", [0, None], ids=["dense", "slots"])
def test_ep_world2_equals_single_process_layer(tmp_path, oracle_lib, skew, capacity):
    """capacity 0: dense blocks sized by an exchange of the counts; None: the
    automatic choice for these 6 home tokens, fixed-capacity slots with
    equal splits and empty slots (id -1)."""
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), skew, capacity, str(tmp_path)), nprocs=world, join=True)
    W, gate, up, down, X = _weights(skew)
    rids, rw, ry = oracle_lib.moe_layer(X, W, gate, up, down, 14, I, K)
    for rank in range(world):
        out = np.load(tmp_path / f"out{rank}.npy")
        ids = np.load(tmp_path / f"ids{rank}.npy")
        assert np.array_equal(ids, rids[rank::world])
        assert np.array_equal(out.view(np.uint32), ry[rank::world].view(np.uint32))
    if skew:
        assert (rids < E // 2).all()      # rank 1 owned no routed expert
