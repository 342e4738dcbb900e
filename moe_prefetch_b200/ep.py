"""Expert-parallel MoE layers for batched decode and prefill.

Rank g of a process group of `world` ranks (one per GPU) owns experts
[g * E / world, (g + 1) * E / world) of every layer; its MoeStack holds only
those, in slots 0 .. E/world - 1.  The router weights are replicated.  One
layer over a rank's home tokens:

  1. route + pack (libmoeb200): ids/w of the home tokens and the pairs in
     owner-rank order, each with its token row and expert id;
  2. all-to-all of the ids and rows (NCCL over NVLink on GPUs): in fixed
     per-rank blocks for small batches, or dense after an exchange of the
     per-rank counts;
  3. the owner runs its experts on the rows it received (grouped GEMV or
     tcgen05 GEMM, unweighted rows);
  4. all-to-all of the rows back, in the order they came;
  5. the home rank combines them in rank order.

With exchange="peer" (ExpertParallelStack on GPUs, world >= 2) steps 2 and
4 are the library's own kernels instead of NCCL: every rank's device memory
holds a mailbox, opened by the other ranks' processes with CUDA IPC; the
pairs are stored straight into the owner's mailbox and the rows straight
back into the home rank's, each followed by a flag the receiver waits for
on the device.  Only routed pairs cross NVLink and nothing waits for the
host, so prefill too can be captured in a CUDA graph.

The reference has no multi-GPU code; the result equals the single-GPU layer
(bit for bit on the GEMV path).  The orchestration works on any
torch.distributed backend: the three device steps come from an `ops` object,
so the exchange logic is testable with gloo on the CPU.
"""
import ctypes as C

import torch
import torch.distributed as dist

from .config import MoeCacheConfig
from .stack import MoeStack, Q4K_BYTES, Q6K_BYTES, _ptr, _stream

PATHS = {"auto": 0, "gemv": 1, "gemm": 2}


def _a2a(out, inp, out_splits, in_splits, group, world):
    if world == 1:
        out.copy_(inp)
    else:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


CAPACITY_MAX_TOKENS = 64   # home tokens up to which the exchange uses fixed-capacity slots


def ep_layer_forward_peer(ops, layer, x, path="auto"):
    """ep_layer_forward over the peer-memory mailboxes (ops: LibEPOps of a
    stack whose mailbox is connected).  path "auto" takes the GEMV for up to
    CAPACITY_MAX_TOKENS home tokens and the GEMM above.  Every rank must
    pass the same number of home tokens (the mailbox blocks of a layer hold
    n_tok * n_used pairs) and the same path (the owners run one path on
    everyone's pairs)."""
    n_tok = x.shape[0]
    if path == "auto":
        path = "gemv" if n_tok <= CAPACITY_MAX_TOKENS else "gemm"
    ids, w, send_count, pos, send_ids, send_x = ops.route_pack(layer, x, ops.world, 0)
    ops.push(n_tok, send_count, send_ids, send_x)
    ops.serve(layer, n_tok, path)
    shared = ops.shared_rows(layer, x, path) if getattr(ops, "n_shared", 0) else None
    out = ops.collect(pos, w, n_tok, shared)
    return out, ids, w


def ep_layer_forward(ops, layer, x, group=None, path="auto", capacity=None):
    """One expert-parallel MoE layer over this rank's home tokens x
    [n_tok, n_embd]; returns (out, ids, w).  Every rank of the group must
    call it for the same layer (the exchange is collective).

    capacity (slots per destination rank; None: automatic) selects the
    exchange.  With capacity slots per rank, every rank's pairs for rank d
    sit in a fixed block and the all-to-alls use equal splits, so nothing
    waits for the host.  The padding moves world * capacity rows.  Without
    it (capacity 0) the blocks are dense, and the send counts travel first
    and are read on the host to size the exchange.  The automatic choice
    takes capacity = n_tok * n_used for up to CAPACITY_MAX_TOKENS home tokens
    (batched decode) or on one rank, and the dense exchange above (prefill).  Every rank must
    pass the same choice.  With capacity slots the "auto" path is the GEMV
    (few pairs per expert), and no step of the layer waits for the host, so
    a sequence of layers can be captured in a CUDA graph."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    n_tok = x.shape[0]
    if capacity is None:   # one rank: every pair stays, no padding and no count exchange
        capacity = n_tok * ops.n_used if n_tok <= CAPACITY_MAX_TOKENS or world == 1 else 0
    if capacity > 0 and world > 1 and path == "auto":
        path = "gemv"   # the padded slots are mostly empty: few pairs per expert
    ids, w, send_count, pos, send_ids, send_x = ops.route_pack(layer, x, world, capacity)
    if capacity > 0:
        recv_ids = torch.empty_like(send_ids)
        recv_x = torch.empty_like(send_x)
        _a2a(recv_ids, send_ids, None, None, group, world)
        _a2a(recv_x, send_x, None, None, group, world)
        y_rows = ops.experts_rows(layer, recv_x, recv_ids, path)
        back = torch.empty_like(y_rows)
        _a2a(back, y_rows, None, None, group, world)
    else:
        recv_count = torch.empty_like(send_count)
        _a2a(recv_count, send_count, None, None, group, world)
        counts = torch.stack([send_count, recv_count]).cpu()
        send_splits = [int(v) for v in counts[0]]
        recv_splits = [int(v) for v in counts[1]]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        recv_ids = torch.empty(n_recv, dtype=send_ids.dtype, device=x.device)
        recv_x = torch.empty(n_recv, x.shape[1], dtype=send_x.dtype, device=x.device)
        _a2a(recv_ids, send_ids[:n_send], recv_splits, send_splits, group, world)
        _a2a(recv_x, send_x[:n_send], recv_splits, send_splits, group, world)
        y_rows = ops.experts_rows(layer, recv_x, recv_ids, path)
        back = torch.empty(n_send, x.shape[1], dtype=y_rows.dtype, device=x.device)
        _a2a(back, y_rows, send_splits, recv_splits, group, world)
    # an always-on shared expert is replicated on every rank: rows of the home tokens
    shared = ops.shared_rows(layer, x, path) if getattr(ops, "n_shared", 0) else None
    out = ops.combine(back, pos, w, n_tok, shared)
    return out, ids, w


class LibEPOps:
    """The three device steps of ep_layer_forward, from libmoeb200.so."""

    def __init__(self, stack, world=1):
        self.st = stack
        self.n_shared = stack.n_shared
        self.n_used = stack.n_used
        self.world = world

    def route_pack(self, layer, x, world, capacity=0):
        st = self.st
        x = x.contiguous()
        n_tok, P = x.shape[0], x.shape[0] * st.n_used
        slots = world * capacity if capacity > 0 else P
        dev = x.device
        ids = torch.empty(n_tok, st.n_used, dtype=torch.int32, device=dev)
        w = torch.empty(n_tok, st.n_used, dtype=torch.float32, device=dev)
        send_count = torch.empty(world, dtype=torch.int32, device=dev)
        pos = torch.empty(P, dtype=torch.int32, device=dev)
        send_ids = torch.empty(slots, dtype=torch.int32, device=dev)
        send_x = torch.empty(slots, st.n_embd, dtype=torch.float32, device=dev)
        st._ck(st.lib.moe_ep_route_pack(st.ctx, layer, _ptr(x), n_tok, world, capacity, _ptr(ids),
                                        _ptr(w), _ptr(send_count), _ptr(pos), _ptr(send_ids),
                                        _ptr(send_x), _stream()), "moe_ep_route_pack")
        return ids, w, send_count, pos, send_ids, send_x

    def experts_rows(self, layer, x_rows, ids, path):
        st = self.st
        y = torch.empty_like(x_rows)
        st._ck(st.lib.moe_experts_rows(st.ctx, layer, _ptr(x_rows), _ptr(ids), x_rows.shape[0],
                                       _ptr(y), PATHS[path], _stream()), "moe_experts_rows")
        return y

    def shared_rows(self, layer, x, path):
        ids = torch.full((x.shape[0],), self.st.n_expert, dtype=torch.int32, device=x.device)
        return self.experts_rows(layer, x.contiguous(), ids, path)

    def push(self, n_tok, send_count, send_ids, send_x):
        st = self.st
        st._ck(st.lib.moe_ep_push(st.ctx, n_tok, _ptr(send_count), _ptr(send_ids), _ptr(send_x), _stream()),
               "moe_ep_push")

    def serve(self, layer, n_tok, path):
        st = self.st
        st._ck(st.lib.moe_ep_serve(st.ctx, layer, n_tok, PATHS[path], _stream()), "moe_ep_serve")

    def collect(self, pos, w, n_tok, add_rows=None):
        st = self.st
        out = torch.empty(n_tok, st.n_embd, dtype=torch.float32, device=w.device)
        st._ck(st.lib.moe_ep_collect(st.ctx, _ptr(pos), _ptr(w), n_tok, _ptr(add_rows), _ptr(out), _stream()),
               "moe_ep_collect")
        return out

    def combine(self, y_rows, pos, w, n_tok, add_rows=None):
        st = self.st
        out = torch.empty(n_tok, st.n_embd, dtype=torch.float32, device=w.device)
        st._ck(st.lib.moe_ep_combine(st.ctx, _ptr(y_rows), _ptr(pos), _ptr(w), n_tok, _ptr(add_rows),
                                     _ptr(out), _stream()), "moe_ep_combine")
        return out


class ExpertParallelStack:
    """The MoE stack of this rank under expert parallelism: its share of the
    experts in slots, the full router, and ep_layer_forward over `group`."""

    def __init__(self, n_layers, n_expert=128, n_used=8, n_embd=2048, n_ff=768, group=None,
                 device=None, n_shared=0, exchange="nccl", max_home_tokens=256):
        """exchange: "nccl" (torch.distributed all-to-all) or "peer" (this
        library's kernels over peer-memory mailboxes; GPUs, world >= 2, up to
        max_home_tokens home tokens per layer)."""
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_expert % self.world:
            raise ValueError(f"{self.world} ranks do not divide {n_expert} experts")
        self.per_rank = n_expert // self.world
        self.e0 = self.rank * self.per_rank
        dev = device if device is not None else torch.cuda.current_device()
        self.st = MoeStack(n_layers, n_expert=n_expert, n_used=n_used, n_embd=n_embd, n_ff=n_ff,
                           cache=MoeCacheConfig(n_slots=self.per_rank), device=dev, n_shared=n_shared)
        self.ops = LibEPOps(self.st, self.world)
        self.exchange = exchange if self.world > 1 else "nccl"
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if self.exchange == "peer":
            self._connect(max_home_tokens)

    def _connect(self, max_home_tokens):
        """Create this rank's mailbox, all-gather the IPC handles, open the
        others'.  A barrier keeps ranks from sending before everyone is
        connected."""
        st = self.st
        h = torch.zeros(64, dtype=torch.uint8)
        st._ck(st.lib.moe_ep_mailbox_create(st.ctx, self.world, self.rank, max_home_tokens, _ptr(h)),
               "moe_ep_mailbox_create")
        hd = h.to(st.device)
        allh = torch.empty(self.world * 64, dtype=torch.uint8, device=st.device)
        dist.all_gather_into_tensor(allh, hd, group=self.group)
        allh = allh.cpu()
        st._ck(st.lib.moe_ep_mailbox_connect(st.ctx, _ptr(allh)), "moe_ep_mailbox_connect")
        torch.cuda.synchronize(st.device)
        dist.barrier(group=self.group)

    def synth(self, seed=0, sigma=0.02, router_sigma=0.02):
        """The weights MoeStack.synth_resident(seed) generates, this rank's
        experts only: each layer's full expert set is generated into a
        temporary buffer and the owned range copied into the slots."""
        st = self.st
        E, per = st.n_expert, self.per_rank
        nbg = E * st.gate_bytes // Q4K_BYTES
        nbd = E * st.down_bytes // Q6K_BYTES
        tmp = torch.empty(E * max(st.gate_bytes, st.down_bytes), dtype=torch.uint8, device=st.device)
        s = _stream()
        for il in range(st.n_layers):
            base = (seed + 1000 * il) & 0xFFFFFFFF
            g, u, d = st.slot_views(il)
            for view, nb, qt, off, nbytes in ((g, nbg, 12, 0, st.gate_bytes), (u, nbg, 12, 1, st.gate_bytes),
                                              (d, nbd, 14, 2, st.down_bytes)):
                st._ck(st.lib.moe_synth_weights(C.c_void_p(tmp.data_ptr()), nb, qt, base + off, sigma, s),
                       "synth")
                view[:per].copy_(tmp[:E * nbytes].view(E, nbytes)[self.e0:self.e0 + per])
            r = torch.empty(E, st.n_embd, device=st.device)
            st._ck(st.lib.moe_synth_f32(_ptr(r), r.numel(), base + 3, router_sigma, s), "synth")
            torch.cuda.synchronize(st.device)
            st.set_router(il, r)
            st.place(il, list(range(self.e0, self.e0 + per)), copy=False)
            if st.n_shared:   # replicated on every rank, seeds as MoeStack.synth_resident
                parts = []
                for off, nbytes, qt in ((4, st.gate_bytes, 12), (5, st.gate_bytes, 12), (6, st.down_bytes, 14)):
                    t = torch.empty(nbytes, dtype=torch.uint8, device=st.device)
                    bb = Q4K_BYTES if qt == 12 else Q6K_BYTES
                    st._ck(st.lib.moe_synth_weights(_ptr(t), nbytes // bb, qt, base + off, sigma, s), "synth")
                    parts.append(t)
                torch.cuda.synchronize(st.device)
                st.set_shared_expert(il, *parts)
        del tmp

    def layer_forward(self, layer, x, path="auto"):
        if self.exchange == "peer":
            return ep_layer_forward_peer(self.ops, layer, x, path)
        return ep_layer_forward(self.ops, layer, x, self.group, path)

    def close(self):
        """With mailboxes: every rank's work done, then free (no rank frees
        memory another may still write)."""
        if self.exchange == "peer" and self.st.ctx:
            torch.cuda.synchronize(self.st.device)
            dist.barrier(group=self.group)
        self.st.close()
