"""Benchmark: Qwen3-30B-A3B Q4_K MoE decode tok/s on B200 (% of HBM roofline).

Workload: the 48-layer MoE-FFN stack, Qwen3-30B-A3B
shapes (hidden 2048, 128 experts, top-8, intermediate 768, Q4_K gate/up, Q6_K
down), batch-1 decode, every expert resident.  One step = one decode of 256
tokens, strictly one token after another (one persistent-kernel launch); the
token inputs are AR(1) hidden states (rho 0.9, RMS-normed); attention is the
identity and the residual adds the MoE output.  Synthetic data: seeded
N(0, 0.02) weights generated and quantised on the device, N(0, 0.02) fp32
routers.  Every token streams 1.23 GB of expert and router weights, far more
than the 126 MB L2, so no step reuses another's weights from L2.

    python bench.py [--gpus N --steps K --warmup W]          # this repo's kernels
    python bench.py --impl reference [...]                    # CPU reference path

With N > 1 (torchrun), each rank decodes its own 256-token stream on its own
GPU (batch-1 decode does not shard: replicas, weak scaling); the time is the
max over ranks.  Rank 0 prints one JSON line.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_LAYERS, N_EXPERT, TOP_K, N_EMBD, N_FF = 48, 128, 8, 2048, 768
GATE_BYTES = N_FF * (N_EMBD // 256) * 144            # 884,736
DOWN_BYTES = N_EMBD * (N_FF // 256) * 210            # 1,290,240
EXPERT_BYTES = 2 * GATE_BYTES + DOWN_BYTES           # 3,059,712
ROUTER_BYTES = N_EXPERT * N_EMBD * 4                 # 1,048,576
XY_BYTES = 2 * N_EMBD * 4                            # layer input + output
LAYER_TOKEN_BYTES = ROUTER_BYTES + TOP_K * EXPERT_BYTES + XY_BYTES   # 25,542,656
METRIC = "Qwen3-30B-A3B Q4_K MoE decode tok/s at 1/2/4/8 B200; % of HBM roofline"


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def capture(step):
    """One CUDA graph of step(), replayed once to check it; None when the
    capture is refused (then the step runs eagerly)."""
    import torch
    g = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(g):
            step()
        g.replay()
        torch.cuda.synchronize()
        return g
    except Exception as e:   # capture unsupported here: eager steps
        print(f"cuda graph capture failed ({type(e).__name__}: {str(e)[:120]}); eager steps",
              file=sys.stderr)
        torch.cuda.synchronize()
        return None


def ar1_states(n_tok, n_embd, seed, rho=0.9):
    rng = np.random.default_rng(seed)
    h = np.empty((n_tok, n_embd), np.float32)
    prev = rng.standard_normal(n_embd)
    for t in range(n_tok):
        prev = rho * prev + np.sqrt(1 - rho * rho) * rng.standard_normal(n_embd)
        h[t] = prev
    return (h / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True))).astype(np.float32)


def config_block(tokens):
    return {
        "workload": "config1: 48-layer Qwen3-30B-A3B MoE-FFN stack, batch-1 decode, "
                    f"{tokens} tokens per step, all 128 experts resident",
        "n_layers": N_LAYERS, "n_expert": N_EXPERT, "top_k": TOP_K, "n_embd": N_EMBD,
        "n_ff": N_FF, "quant": "Q4_K gate/up, Q6_K down, Q8_1 activations",
        "tokens_per_step": tokens,
        "l2": "inputs larger than L2: 1.23 GB of expert+router weights per token",
        "parallelism": "replicas (batch-1 decode does not shard)",
    }


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id=None):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = []
        if self.path and os.path.exists(self.path):
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    if self.bus_id and self.bus_id[-12:] not in parts[0].lower():
                        continue
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle's restatement of the ggml CPU rows path
# ---------------------------------------------------------------------------
def cpu_baseline(host_layers, seconds, threads):
    """Times the integer-dot CPU rows path (Q8_K activations, ggml op order,
    OpenMP) on a bounded sample: the given layers' weights, tokens cycled
    through them until `seconds` of CPU work; returns tok/s of the 48-layer
    stack (layer-token rate / 48)."""
    import oracle
    oracle.build()
    rng = np.random.default_rng(5)
    x = ar1_states(64, N_EMBD, 77)
    n = 0
    t0 = time.perf_counter()
    while True:
        L = host_layers[n % len(host_layers)]
        oracle.moe_layer_cpu_fast(x[n % 64], L["router"], L["gate"], L["up"], L["down"], 14,
                                  N_FF, TOP_K, n_threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 8:
            break
    del rng
    return n / el / N_LAYERS, n, el


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    oracle.build()
    threads = host_threads()
    # two layers of weights generated on the host (numpy N(0, 0.02), the
    # oracle's quantiser); the reference's own CPU path cannot be built here
    layers = []
    for il in range(2):
        rng = np.random.default_rng(1000 * il)
        layers.append({
            "gate": oracle.quantize((rng.standard_normal((N_EXPERT * N_FF, N_EMBD)) * 0.02)
                                    .astype(np.float32), 12).reshape(N_EXPERT, -1),
            "up": oracle.quantize((rng.standard_normal((N_EXPERT * N_FF, N_EMBD)) * 0.02)
                                  .astype(np.float32), 12).reshape(N_EXPERT, -1),
            "down": oracle.quantize((rng.standard_normal((N_EXPERT * N_EMBD, N_FF)) * 0.02)
                                    .astype(np.float32), 14).reshape(N_EXPERT, -1),
            "router": (rng.standard_normal((N_EXPERT, N_EMBD)) * 0.02).astype(np.float32),
        })
    per_step = max(1.0, float(args.ref_seconds))
    for _ in range(args.warmup):
        cpu_baseline(layers, min(per_step, 1.0), threads)
    vals, tot_n, tot_t = [], 0, 0.0
    for _ in range(args.steps):
        v, n, el = cpu_baseline(layers, per_step, threads)
        vals.append(v)
        tot_n += n
        tot_t += el
    value = tot_n / tot_t / N_LAYERS
    sample = (f"{tot_n} layer-tokens over 2 host-resident layers (2 x 392 MB), "
              f"{per_step:.0f} s per step; tok/s = layer-tokens/s / 48")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot_t / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": config_block(args.tokens),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's CPU MoE path (ggml mul_mat_id / GGML_OP_MOE_ROWS in patches "
                "against llama.cpp) cannot be built here; this is the oracle's restatement of "
                "it (Q4_K/Q6_K x Q8_K integer dots, ggml op order, OpenMP)",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# config 2: the constrained slot cache, swept over slot budgets and delta
# ---------------------------------------------------------------------------
SWEEP_SLOTS = (16, 32, 56, 96)
SWEEP_DELTA = (0.0, 0.01)
MISS_GRID = (8, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128)


def lru_miss_rates(ids, grid):
    """Per-layer miss rate of an all-admit LRU cache of each size in `grid`
    over a route trace ids [T][L][k]: {size: [rate per layer]}.  Used only to
    rank layers for the byte-priced profile."""
    T, L, K = ids.shape
    out = {g: [0.0] * L for g in grid}
    for il in range(L):
        seq = ids[:, il, :]
        for g in grid:
            last, clock, miss = {}, 0, 0
            for t in range(T):
                for e in seq[t]:
                    clock += 1
                    if e in last:
                        last[e] = clock
                        continue
                    miss += 1
                    if len(last) >= g:
                        del last[min(last, key=last.get)]
                    last[e] = clock
            out[g][il] = miss / float(T * K)
    return out


def run_stream(args):
    """Just-in-time streaming (LLAMA_MOE_STREAM) measured: the config-2 stack
    (48 layers, every expert in pinned host memory, a byte-priced 56-slot
    profile, window admission, early issue, delta 0) decoded token by token
    through the per-layer entry point moe_layer_forward, the next layer's
    input being the RMS-normed residual sum.  The rest of a transformer layer
    (attention) is stood in for by a fixed spin of --attn-us on the GPU per
    layer (torch.cuda._sleep), the time in which streamed copies land.  One
    JSON line per (attention time, streaming off/on)."""
    import torch
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    from moe_prefetch_b200.config import format_slot_profile, greedy_allocate_bytes

    torch.cuda.set_device(0)
    n_layers = args.layers
    warm, timed = args.c2_warm, args.c2_tokens
    res = MoeStack(n_layers=n_layers)
    res.synth_resident(seed=11, keep_router=True)
    host = []
    for il in range(n_layers):
        g, u, d = res.slot_views(il)
        hl = []
        for v in (g, u, d):
            t = torch.empty(N_EXPERT * v.shape[1], dtype=torch.uint8, pin_memory=True)
            t.view(N_EXPERT, -1).copy_(v[:N_EXPERT])
            hl.append(t)
        host.append(tuple(hl))
    routers = [r.clone() for r in res.routers]
    h_trace = torch.from_numpy(ar1_states(256, N_EMBD, seed=4242)).cuda()
    _, dm = res.decode(h_trace, debug=True)
    res.sync()
    trace = dm["ids"].cpu().numpy()
    del dm
    res.close()
    torch.cuda.synchronize()
    miss8 = lru_miss_rates(trace, MISS_GRID)
    grid = [g for g in MISS_GRID if g <= N_EXPERT]
    caps, _, _ = greedy_allocate_bytes(miss8, grid, n_layers, 56, [], [EXPERT_BYTES] * n_layers)
    h = torch.from_numpy(ar1_states(warm + timed, N_EMBD, seed=12345)).cuda()
    # GPU clock cycles for the attention stand-in, from the measured SM clock
    try:
        mhz = int(torch.cuda.clock_rate()) or 1965
    except Exception:   # no NVML: the B200's maximum SM clock
        mhz = 1965
    stream = torch.cuda.current_stream()
    for attn_us in args.attn_us:
        cycles = int(attn_us * mhz)
        for on in (False, True):
            cfg = MoeCacheConfig(n_slots=56, max_inserts=2, admit="window", admit_window=8,
                                 batch_tables=True, early_issue=True, stream=on,
                                 slot_profile=format_slot_profile(caps))
            st = MoeStack(n_layers=n_layers, cache=cfg)
            for il in range(n_layers):
                st.set_router(il, routers[il])
                st.set_expert_weights(il, *host[il])

            def token(t):
                x = h[t:t + 1]
                for il in range(n_layers):
                    if cycles:
                        torch.cuda._sleep(cycles)
                    y, _, _ = st.layer_forward(il, x)
                    z = x + y
                    x = z * torch.rsqrt((z * z).mean(-1, keepdim=True) + 1e-6)
                st.step()
            for t in range(warm):
                token(t)
            torch.cuda.synchronize()
            s0, q0 = st.stats(), st.stream_stats()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for t in range(warm, warm + timed):
                token(t)
            e1.record(stream)
            torch.cuda.synchronize()
            s1, q1 = st.stats(), st.stream_stats()
            ms = e0.elapsed_time(e1)
            d = {k: s1[k] - s0[k] for k in s1}
            q = {k: q1[k] - q0[k] for k in q1}
            routed = d["hits"] + d["misses"]
            line = {
                "metric": "config2 per-layer decode with just-in-time streaming", "value": timed / (ms / 1000.0),
                "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
                "config": {"workload": "config2 stack through moe_layer_forward, one token at a time, "
                                       "56-slot byte-priced profile, window admission, early issue, delta 0",
                           "stream": on, "attention_stand_in_us": attn_us,
                           "warm_tokens": warm, "timed_tokens": timed},
                "hit_rate": d["hits"] / routed if routed else None,
                "misses_per_token": d["misses"] / timed,
                "ms_per_token": ms / timed,
                "stream": ({"experts_streamed_per_token": q["words"] / timed,
                            "in_time_per_token": q["in_time"] / timed,
                            "late_per_token": q["late"] / timed,
                            "dropped_late_per_token": q["dropped_late"] / timed,
                            "given_back_per_token": q["given_back"] / timed,
                            "stream_gbs": q["bytes"] / (ms / 1000.0) / 1e9} if on else None),
            }
            print(json.dumps(line), flush=True)
            st.close()
    return 0


def run_config2(args):
    """Config 2: the 48-layer stack with every expert in pinned host memory
    and a slot cache of n_slots per layer (byte-priced per-layer profile from
    a route trace of a separate token stream), second-miss admission (window
    8), batched table writes, delta in {0, 0.01}.  Batch-1 decode token by
    token with the cache step between tokens; misses are read zero-copy and
    admitted experts uploaded on the copy stream.  One JSON line per point."""
    import torch
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    from moe_prefetch_b200.config import format_slot_profile, greedy_allocate_bytes

    torch.cuda.set_device(0)
    n_layers = args.layers
    warm, timed = args.c2_warm, args.c2_tokens
    res = MoeStack(n_layers=n_layers)
    res.synth_resident(seed=11, keep_router=True)
    host = []
    for il in range(n_layers):
        g, u, d = res.slot_views(il)
        hl = []
        for v in (g, u, d):
            t = torch.empty(N_EXPERT * v.shape[1], dtype=torch.uint8, pin_memory=True)
            t.view(N_EXPERT, -1).copy_(v[:N_EXPERT])
            hl.append(t)
        host.append(tuple(hl))
    routers = [r.clone() for r in res.routers]
    # route trace on a separate stream of tokens (delta 0: routing does not
    # depend on the cache) -> per-layer miss curves -> byte-priced profiles
    h_trace = torch.from_numpy(ar1_states(256, N_EMBD, seed=4242)).cuda()
    _, dm = res.decode(h_trace, debug=True)
    res.sync()
    trace = dm["ids"].cpu().numpy()
    del dm
    res.close()
    torch.cuda.synchronize()
    miss8 = lru_miss_rates(trace, MISS_GRID)
    h = torch.from_numpy(ar1_states(warm + timed, N_EMBD, seed=12345)).cuda()
    out = torch.empty_like(h)
    stream = torch.cuda.current_stream()
    for ns in SWEEP_SLOTS:
        grid = [g for g in MISS_GRID if g <= N_EXPERT]
        caps, used, budget = greedy_allocate_bytes(miss8, grid, n_layers, ns, [],
                                                   [EXPERT_BYTES] * n_layers)
        for delta in SWEEP_DELTA:
            cfg = MoeCacheConfig(n_slots=ns, max_inserts=2, admit="window", admit_window=8,
                                 batch_tables=True, cache_prior=delta,
                                 slot_profile=format_slot_profile(caps))
            st = MoeStack(n_layers=n_layers, cache=cfg)
            for il in range(n_layers):
                st.set_router(il, routers[il])
                st.set_expert_weights(il, *host[il])
            for t in range(warm):
                st.decode(h[t:t + 1], out[t:t + 1])
                st.step()
            st.sync()
            s0 = st.stats()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for t in range(warm, warm + timed):
                st.decode(h[t:t + 1], out[t:t + 1])
                st.step()
            e1.record(stream)
            torch.cuda.synchronize()
            st.sync()
            s1 = st.stats()
            ms = e0.elapsed_time(e1)
            d = {k: s1[k] - s0[k] for k in s1}
            routed = d["hits"] + d["misses"]
            line = {
                "metric": "config2 slot-cache decode", "value": timed / (ms / 1000.0),
                "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
                "config": {"workload": "config2: 48-layer stack, experts in pinned host memory, "
                                       "slot cache, window admission (W=8), batched tables",
                           "n_slots": ns, "delta": delta, "max_inserts": 2,
                           "profile": "byte-priced greedy from a 256-token route trace "
                                      "(separate seed)",
                           "slots_total": int(sum(caps)), "slots_uniform_total": ns * n_layers,
                           "warm_tokens": warm, "timed_tokens": timed},
                "hit_rate": d["hits"] / routed if routed else None,
                "misses_per_token": d["misses"] / timed,
                # step-scheduled uploads; "uploads" counts only the early-issue path
                "uploads_per_token": d["scheduled"] / timed,
                "published_per_token": d["published"] / timed,
                "upload_gbs": d["upload_bytes"] / (ms / 1000.0) / 1e9,
                # while the copy stream runs the uploads (the host link's share)
                "upload_gbs_during_copies": (d["upload_bytes"] / d["upload_ns"] if d["upload_ns"] else None),
                "zero_copy_miss_gbs": d["misses"] * EXPERT_BYTES / (ms / 1000.0) / 1e9,
                "ms_per_token": ms / timed,
            }
            print(json.dumps(line), flush=True)
            st.close()
            torch.cuda.synchronize()
    return 0


# ---------------------------------------------------------------------------
# config 3: batched decode and prefill, expert-parallel over the ranks
# ---------------------------------------------------------------------------
def ep_measure(world, rank, n_layers, dec_steps, pre_chunks, warmup, exchange="peer"):
    """The config-3 expert-parallel workloads on the ranks of the current
    process group (or one GPU): rank g owns experts [g E/N, (g+1) E/N) of
    every layer.  The dispatch and combine go through the library's
    peer-memory mailboxes (exchange "peer", the default) or NCCL all-to-all
    ("nccl").  32 sequences decoding (32 / N home tokens per rank per step)
    and one 512-token prefill chunk (512 / N per rank); with the mailboxes
    both whole steps replay as CUDA graphs (with NCCL only the decode step,
    whose fixed-capacity exchange does not wait for the host).  Inputs are
    i.i.d. N(0, 1) RMS-normed rows.  Total work is fixed as N grows (strong
    scaling).  Device time is CUDA events on each rank, max over ranks.
    Returns the JSON lines (every rank computes them)."""
    import torch
    import torch.distributed as dist
    from moe_prefetch_b200.ep import ExpertParallelStack

    ep = ExpertParallelStack(n_layers, exchange=exchange, max_home_tokens=max(512 // world, 32))
    exchange = ep.exchange   # one GPU: no exchange
    ep.synth(seed=11)
    stream = torch.cuda.current_stream()

    def rows(n, seed):
        rng = np.random.default_rng(seed)
        h = rng.standard_normal((n, N_EMBD))
        return (h / np.sqrt((h ** 2).mean(-1, keepdims=True))).astype(np.float32)

    def timed(x, steps, warm, path, graph):
        def step():
            for il in range(n_layers):
                ep.layer_forward(il, x, path)
        for _ in range(warm):
            step()
        g = None
        if graph:   # nothing in the step waits for the host: it replays as one CUDA graph
            torch.cuda.synchronize()
            g = capture(step)
        used_graph[0] = g is not None
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            if g is not None:
                g.replay()
            else:
                step()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g   # a graph holding NCCL calls goes before the process group
        return float(t[0])

    used_graph = [False]
    lines = []
    dec_seqs = 32
    if dec_seqs % world == 0:
        x = torch.from_numpy(rows(dec_seqs, 500)[rank::world].copy()).cuda()
        ms = timed(x, dec_steps, warmup, "auto", graph=True)
        xpath = "peer-memory mailboxes" if exchange == "peer" else "NCCL fixed-capacity all-to-all"
        lines.append({
            "metric": "config3 expert-parallel batched decode", "value": dec_seqs * dec_steps / (ms / 1e3),
            "unit": "tok/s", "n_gpus": world, "steps": dec_steps, "warmup": warmup,
            "ms_per_step": ms / dec_steps, "higher_is_better": True, "scaling": "strong",
            "config": {"workload": f"config3 decode: {dec_seqs} sequences x {dec_steps} steps, "
                                   f"{n_layers} layers, EP {N_EXPERT // world} experts/GPU",
                       "path": f"grouped GEMV, {xpath if world > 1 else 'no exchange'}",
                       "cuda_graph": used_graph[0], "data": "synthetic"}})
    pre_tok = 512
    if pre_tok % world == 0:
        x = torch.from_numpy(rows(pre_tok, 501)[rank::world].copy()).cuda()
        ms = timed(x, pre_chunks, max(1, warmup), "auto", graph=exchange == "peer" or world == 1)
        flops = 2.0 * pre_tok * TOP_K * 3 * N_EMBD * N_FF * n_layers * pre_chunks
        lines.append({
            "metric": "config3 expert-parallel prefill", "value": pre_tok * pre_chunks / (ms / 1e3),
            "unit": "tok/s", "n_gpus": world, "steps": pre_chunks, "warmup": max(1, warmup),
            "ms_per_step": ms / pre_chunks, "higher_is_better": True, "scaling": "strong",
            "expert_tflops_whole_job": flops / (ms / 1e3) / 1e12,
            "config": {"workload": f"config3 prefill: one {pre_tok}-token chunk per step, "
                                   f"{n_layers} layers, EP {N_EXPERT // world} experts/GPU",
                       "path": "tcgen05 grouped GEMM, " + (("peer-memory mailboxes" if exchange == "peer"
                                                           else "NCCL all-to-all sized on the host")
                                                          if world > 1 else "no exchange"),
                       "cuda_graph": used_graph[0], "data": "synthetic"}})
    ep.close()
    torch.cuda.synchronize()
    return lines


def run_config3(args):
    """Config 3 on its own: ep_measure, one JSON line per workload from rank 0."""
    import datetime
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    lines = ep_measure(world, rank, args.layers, args.c3_decode_steps, args.c3_prefill_chunks,
                       args.warmup, args.ep_exchange)
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# config 4: 256 experts, n_ff 512, one always-on shared expert, 40 layers
# ---------------------------------------------------------------------------
C4_LAYERS, C4_EXPERT, C4_FF = 40, 256, 512
C4_EXPERT_BYTES = 2 * C4_FF * (N_EMBD // 256) * 144 + N_EMBD * (C4_FF // 256) * 210   # 2,039,808
C4_LAYER_TOKEN_BYTES = C4_EXPERT * N_EMBD * 4 + (TOP_K + 1) * C4_EXPERT_BYTES + XY_BYTES


def run_config4(args):
    """Config 4: 40 layers of 256 routed experts (top-8, n_ff 512) plus one
    always-on shared expert.  At N = 1: (a) resident batch-1 decode (one
    persistent launch per step) with its HBM roofline; (b) batch-1 decode
    through a 96-slot cache, delta 0.01, experts in pinned host memory, window
    admission, token by token with the cache step between tokens.  At every N:
    (c) 32-sequence expert-parallel decode (the shared expert replicated).
    One JSON line per measurement from rank 0."""
    import datetime
    import torch
    import torch.distributed as dist
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    from moe_prefetch_b200.ep import ExpertParallelStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    L = C4_LAYERS
    stream = torch.cuda.current_stream()
    lines = []
    cfg_base = {"n_layers": L, "n_expert": C4_EXPERT, "top_k": TOP_K, "n_ff": C4_FF, "n_shared": 1,
                "quant": "Q4_K gate/up, Q6_K down", "data": "synthetic"}
    if world == 1:
        # (a) resident decode
        tokens = 128
        st = MoeStack(n_layers=L, n_expert=C4_EXPERT, n_ff=C4_FF, n_shared=1,
                      cache=MoeCacheConfig(cache_prior=0.01))
        st.synth_resident(seed=17, keep_router=True)
        h = torch.from_numpy(ar1_states(tokens, N_EMBD, seed=321)).cuda()
        out = torch.empty_like(h)
        for _ in range(args.warmup):
            st.decode(h, out)
        st.sync()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        steps = max(3, args.steps // 4)
        e0.record(stream)
        for _ in range(steps):
            st.decode(h, out)
        e1.record(stream)
        torch.cuda.synchronize()
        st.sync()
        ms = e0.elapsed_time(e1) / steps
        peak, peak_kind = measured_peaks()
        achieved = C4_LAYER_TOKEN_BYTES * L * tokens / (ms / 1e3) / 1e9
        lines.append({"metric": "config4 batch-1 decode, all experts resident", "value": tokens / (ms / 1e3),
                      "unit": "tok/s", "n_gpus": 1, "steps": steps, "ms_per_step": ms,
                      "higher_is_better": True,
                      "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                   "frac": achieved / peak, "peak_kind": peak_kind,
                                   "algorithmic_bytes_per_layer_token": C4_LAYER_TOKEN_BYTES},
                      "config": dict(cfg_base, workload=f"config4 resident decode, {tokens} tokens per step")})
        # (b) 96-slot cache, delta 0.01: host copies of every layer's experts
        host = []
        for il in range(L):
            g, u, d = st.slot_views(il)
            hl = []
            for v in (g, u, d):
                t = torch.empty(C4_EXPERT * v.shape[1], dtype=torch.uint8, pin_memory=True)
                t.view(C4_EXPERT, -1).copy_(v[:C4_EXPERT])
                hl.append(t)
            host.append(tuple(hl))
        routers = [r.clone() for r in st.routers]
        shared = [tuple(p.clone() for p in sp) for sp in st.shared]
        st.close()
        torch.cuda.synchronize()
        warm, timed = args.c2_warm, args.c2_tokens
        cc = MoeStack(n_layers=L, n_expert=C4_EXPERT, n_ff=C4_FF, n_shared=1,
                      cache=MoeCacheConfig(n_slots=96, max_inserts=2, admit="window", admit_window=8,
                                           batch_tables=True, cache_prior=0.01))
        for il in range(L):
            cc.set_router(il, routers[il])
            cc.set_expert_weights(il, *host[il])
            cc.set_shared_expert(il, *shared[il])
        hc = torch.from_numpy(ar1_states(warm + timed, N_EMBD, seed=654)).cuda()
        oc = torch.empty_like(hc)
        for t in range(warm):
            cc.decode(hc[t:t + 1], oc[t:t + 1])
            cc.step()
        cc.sync()
        s0 = cc.stats()
        e0.record(stream)
        for t in range(warm, warm + timed):
            cc.decode(hc[t:t + 1], oc[t:t + 1])
            cc.step()
        e1.record(stream)
        torch.cuda.synchronize()
        cc.sync()
        s1 = cc.stats()
        ms = e0.elapsed_time(e1)
        d = {k: s1[k] - s0[k] for k in s1}
        routed = d["hits"] + d["misses"]
        lines.append({"metric": "config4 batch-1 decode, 96-slot cache, delta 0.01",
                      "value": timed / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
                      "hit_rate": d["hits"] / routed if routed else None,
                      "uploads_per_token": d["scheduled"] / timed,
                      "upload_gbs": d["upload_bytes"] / (ms / 1e3) / 1e9,
                      "zero_copy_miss_gbs": d["misses"] * C4_EXPERT_BYTES / (ms / 1e3) / 1e9,
                      "ms_per_token": ms / timed,
                      "config": dict(cfg_base, workload="config4 cache decode: 96 slots/layer, window "
                                                        "admission W=8, batched tables",
                                     warm_tokens=warm, timed_tokens=timed)})
        cc.close()
        del host
        torch.cuda.synchronize()
    # (c) 32-sequence expert-parallel decode
    seqs, steps = 32, args.c3_decode_steps
    if seqs % world == 0 and C4_EXPERT % world == 0:
        ep = ExpertParallelStack(L, n_expert=C4_EXPERT, n_ff=C4_FF, n_shared=1)
        ep.synth(seed=17)
        rng = np.random.default_rng(502)
        xx = rng.standard_normal((seqs, N_EMBD))
        xx = (xx / np.sqrt((xx ** 2).mean(-1, keepdims=True))).astype(np.float32)
        x = torch.from_numpy(xx[rank::world].copy()).cuda()

        def step():
            for il in range(L):
                ep.layer_forward(il, x, "auto")
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        g = capture(step)   # fixed-capacity exchange: one graph per step
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            if g is not None:
                g.replay()
            else:
                step()
        e1.record(stream)
        torch.cuda.synchronize()
        graphed = g is not None
        del g
        t = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        lines.append({"metric": "config4 expert-parallel batched decode", "value": seqs * steps / (ms / 1e3),
                      "unit": "tok/s", "n_gpus": world, "steps": steps, "ms_per_step": ms / steps,
                      "higher_is_better": True, "scaling": "strong",
                      "config": dict(cfg_base, workload=f"config4 decode: {seqs} sequences x {steps} steps, "
                                                        f"EP {C4_EXPERT // world} experts/GPU, shared replicated",
                                     cuda_graph=graphed)})
        ep.close()
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# one layer through one expert path (the profiling case of the batched kernels)
# ---------------------------------------------------------------------------
def run_layer(args):
    """One resident 128-expert layer (config-0 shapes), --tokens RMS-normed
    tokens through moe_layer_forward_path(--path), --warmup untimed calls,
    then --steps timed calls (CUDA events).  One JSON line: us per layer."""
    import torch
    from moe_prefetch_b200 import MoeStack
    torch.cuda.set_device(0)
    st = MoeStack(n_layers=1)
    st.synth_resident(seed=5)
    h = np.random.default_rng(1).standard_normal((args.tokens, N_EMBD))
    x = torch.from_numpy((h / np.sqrt((h ** 2).mean(-1, keepdims=True))).astype(np.float32)).cuda()
    for _ in range(args.warmup):
        st.layer_forward_path(0, x, args.path)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        st.layer_forward_path(0, x, args.path)
    e1.record()
    torch.cuda.synchronize()
    st.sync()
    us = e0.elapsed_time(e1) * 1000.0 / max(args.steps, 1)
    print(json.dumps({"metric": "one MoE layer", "value": us, "unit": "us/layer", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                      "config": {"workload": f"1 layer, {args.tokens} tokens, path {args.path}",
                                 "n_expert": N_EXPERT, "n_ff": N_FF, "data": "synthetic"}}),
          flush=True)
    st.close()
    return 0


# ---------------------------------------------------------------------------
# config 0: one layer, 64 single-token forwards, L2 defeated
# ---------------------------------------------------------------------------
def run_config0(args):
    """Config 0: the single Qwen3-30B-A3B-shape layer (all 128 experts
    resident, delta 0), 64 RMS-normed N(0, 1) inputs, one token per forward.
    L2 reuse is defeated by rotating 8 device copies of the layer (the same
    weights and router in 8 places, 8 x 392 MB): forward t runs on copy t mod
    8, so no forward finds the previous seven's bytes in the 126 MB L2.
    Two arms, CUDA events around all 64 forwards after --warmup rounds:
    - operator: moe_layer_forward per token (the per-layer entry point that
      replaces build_moe_ffn's expert chain: the router on an 8-CTA cluster,
      then the grouped expert kernels), and beside it the allocation-free
      entry point (the same router, the per-pair kernels);
    - persistent: moe_decode over the 8 copies and 8 tokens, i.e. 64
      layer-token forwards in one launch (the copies' inputs are then the
      residual stream instead of fresh rows: the same bytes and arithmetic
      per forward).
    The CPU baseline is the oracle's integer-dot CPU path on the same layer
    (all host threads, a 10 s sample).  One JSON line."""
    import torch
    from moe_prefetch_b200 import MoeStack
    torch.cuda.set_device(0)
    copies = 8
    st = MoeStack(n_layers=copies)
    st.synth_resident(seed=7, keep_router=True)
    g0, u0, d0 = st.slot_views(0)
    for il in range(1, copies):
        g, u, d = st.slot_views(il)
        g.copy_(g0); u.copy_(u0); d.copy_(d0)
        st.set_router(il, st.routers[0])
    torch.cuda.synchronize()
    rng = np.random.default_rng(12345)
    h = rng.standard_normal((64, N_EMBD))
    x = torch.from_numpy((h / np.sqrt((h ** 2).mean(-1, keepdims=True))).astype(np.float32)).cuda()
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def op_round():
        for t in range(64):
            st.layer_forward(t % copies, x[t:t + 1])
    for _ in range(max(args.warmup, 1)):
        op_round()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record()
    op_round()
    e1.record()
    torch.cuda.synchronize()
    us_op = e0.elapsed_time(e1) * 1000.0 / 64
    # the allocation-free entry point: the per-pair kernels
    y1 = torch.empty_like(x[:1])

    def na_round():
        for t in range(64):
            st.layer_forward_noalloc(t % copies, x[t:t + 1], y1)
    na_round()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record()
    na_round()
    e1.record()
    torch.cuda.synchronize()
    us_na = e0.elapsed_time(e1) * 1000.0 / 64
    xd = x[:copies].contiguous()          # 8 tokens x 8 copies = 64 forwards
    out = torch.empty_like(xd)
    for _ in range(max(args.warmup, 1)):
        st.decode(xd, out)
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record()
    st.decode(xd, out)
    e1.record()
    torch.cuda.synchronize()
    st.sync()
    us_dec = e0.elapsed_time(e1) * 1000.0 / 64
    peak, peak_kind = measured_peaks()
    frac = lambda us: LAYER_TOKEN_BYTES / (us * 1e-6) / 1e9 / peak
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        gate, up, down = (v[:N_EXPERT].cpu().numpy() for v in (g0, u0, d0))
        W = st.routers[0].cpu().numpy()
        xs = x.cpu().numpy()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            oracle.moe_layer_cpu_fast(xs[n % 64], W, gate, up, down, 14, N_FF, TOP_K,
                                      n_threads=os.cpu_count())
            n += 1
        cpu = {"value": n / (time.perf_counter() - t0), "unit": "forwards/s", "cores": os.cpu_count(),
               "kind": "port", "sample": f"{n} single-token forwards of the layer (10 s)"}
    st.close()
    print(json.dumps({
        "metric": "config0 single-layer batch-1 forward", "value": 1e6 / us_dec, "unit": "forwards/s",
        "n_gpus": 1, "steps": 64, "warmup": max(args.warmup, 1), "higher_is_better": True,
        "us_per_forward": {"persistent": us_dec, "operator": us_op, "operator_noalloc_per_pair": us_na},
        "operator_forwards_per_s": 1e6 / us_op,
        "roofline": {"bound": "hbm", "unit": "GB/s", "peak": peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_forward": LAYER_TOKEN_BYTES,
                     "frac_persistent": frac(us_dec), "frac_operator": frac(us_op)},
        "cpu_baseline": cpu,
        "config": {"workload": "config0: 1 layer x 64 single-token forwards, all 128 experts resident, delta 0",
                   "l2": "defeated: 8 device copies of the layer in rotation (8 x 392 MB)",
                   "data": "synthetic (seeded N(0,0.02) weights quantised on device; N(0,1) RMS-normed inputs)"}}),
        flush=True)
    return 0


# ---------------------------------------------------------------------------
# the host link: the denominators of config 2's upload and zero-copy rates
# ---------------------------------------------------------------------------
def run_hostlink(args):
    """Host-link peaks on this box, and the library's own rates against them.
    (1) one 1 GiB pinned host -> device cudaMemcpyAsync on a dedicated
    non-blocking stream (the copy engine's peak); (2) the uploader's pattern:
    64 expert jobs of three copies (gate, up, down slices) from pinned host
    memory, back to back on that stream; (3) zero-copy reads by the decode
    kernel: a frozen cache that holds nothing, so that every routed expert of
    every layer is read from registered host memory (--layers x --tokens
    layer-tokens, 8 experts each).  One JSON line."""
    import torch
    from moe_prefetch_b200 import MoeCacheConfig, MoeStack
    torch.cuda.set_device(0)
    cs = torch.cuda.Stream(priority=0)

    def copy_rate(dst, src_views, reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        nbytes = 0
        with torch.cuda.stream(cs):
            for d, v in src_views:               # warm-up
                d.copy_(v, non_blocking=True)
            e0.record(cs)
            for _ in range(reps):
                for d, v in src_views:
                    d.copy_(v, non_blocking=True)
                    nbytes += v.numel()
            e1.record(cs)
        cs.synchronize()
        return nbytes / (e0.elapsed_time(e1) / 1000.0) / 1e9

    big = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    dbig = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    peak = copy_rate(dbig, [(dbig, big)], 5)
    del big, dbig
    gb, db = GATE_BYTES, DOWN_BYTES
    n_jobs = 64
    hs = torch.empty(n_jobs * (2 * gb + db), dtype=torch.uint8, pin_memory=True)
    ds = torch.empty_like(hs, device="cuda")
    views = []
    for j in range(n_jobs):
        o = j * (2 * gb + db)
        for a, n in ((o, gb), (o + gb, gb), (o + 2 * gb, db)):
            views.append((ds[a:a + n], hs[a:a + n]))
    jobs = copy_rate(None, views, 4)
    del hs, ds
    torch.cuda.synchronize()
    # zero-copy: every expert host-resident, nothing admitted
    L, T = args.layers, args.tokens
    res = MoeStack(n_layers=L)
    res.synth_resident(seed=11, keep_router=True)
    host = []
    for il in range(L):
        g, u, d = res.slot_views(il)
        hl = []
        for v in (g, u, d):
            t = torch.empty(N_EXPERT * v.shape[1], dtype=torch.uint8, pin_memory=True)
            t.view(N_EXPERT, -1).copy_(v[:N_EXPERT])
            hl.append(t)
        host.append(tuple(hl))
    routers = [r.clone() for r in res.routers]
    res.close()
    torch.cuda.synchronize()
    st = MoeStack(n_layers=L, cache=MoeCacheConfig(n_slots=8, freeze=True))
    for il in range(L):
        st.set_router(il, routers[il])
        st.set_expert_weights(il, *host[il])
    h = torch.from_numpy(ar1_states(T, N_EMBD, seed=5)).cuda()
    out = torch.empty_like(h)
    st.decode(h, out)
    st.sync()
    s0 = st.stats()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    st.decode(h, out)
    e1.record()
    torch.cuda.synchronize()
    st.sync()
    s1 = st.stats()
    ms = e0.elapsed_time(e1)
    misses = s1["misses"] - s0["misses"]
    zc = misses * EXPERT_BYTES / (ms / 1000.0) / 1e9
    st.close()
    print(json.dumps({
        "metric": "host link", "unit": "GB/s",
        "pinned_h2d_1GiB_gbs": peak, "upload_pattern_gbs": jobs,
        "upload_pattern_frac": jobs / peak,
        "decode_zero_copy_gbs": zc, "decode_zero_copy_frac": zc / peak,
        "zero_copy_layer_tokens": L * T, "zero_copy_misses": misses,
        "config": {"workload": "pinned copies on a dedicated stream; decode with every expert in host memory",
                   "upload_jobs": n_jobs, "expert_bytes": EXPERT_BYTES, "layers": L, "tokens": T,
                   "data": "synthetic"}}), flush=True)
    return 0


# ---------------------------------------------------------------------------
# where a decode layer's time goes (the kernel's own phase stamps)
# ---------------------------------------------------------------------------
PHASES = [(0, 1, "grid barrier A"), (1, 2, "router totals"), (2, 6, "selection"),
          (6, 7, "copy issue (warp 0)"), (6, 8, "gate/up rows done (warp 1)"),
          (8, 9, "rank signals"), (9, 10, "rank 0: wait, activations -> Q8_1, down rows"),
          (10, 11, "other ranks + combine")]


def run_phases(args):
    """Config-1 shapes (or config 4 with --c4), --layers x --tokens AR(1)
    tokens through one moe_decode launch with phase stamps (%globaltimer, one
    per CTA per phase boundary); prints per phase the median over CTAs and
    layer-tokens (the first token's layers skipped), the median of the
    per-layer-token maximum over CTAs, and the layer time."""
    import ctypes as C
    import torch
    from moe_prefetch_b200 import MoeStack
    from moe_prefetch_b200._lib import MoeDecodeDbg
    torch.cuda.set_device(0)
    L, T, PH = args.layers, args.tokens, 12
    kw = dict(n_expert=256, n_ff=512, n_shared=1) if args.c4 else {}
    st = MoeStack(n_layers=L, **kw)
    st.synth_resident(seed=3)
    h = torch.from_numpy(ar1_states(T, N_EMBD, 5)).cuda()
    out = torch.empty_like(h)
    for _ in range(max(args.warmup, 1)):
        st.decode(h, out)
    st.sync()
    G = st.decode_info()["grid"]
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    # spec 0: gate/up copies issued from the logits' top-k before the exact
    # selection (the default); 1: issued after it
    for spec in (0, 1):
        prof = torch.zeros(T, L, PH, G, dtype=torch.int64, device="cuda")
        dbg = MoeDecodeDbg(None, None, None, None, prof.data_ptr(), 0, spec)
        rc = st.lib.moe_decode(st.ctx, C.c_void_p(h.data_ptr()), C.c_void_p(out.data_ptr()), T, C.byref(dbg),
                               s)
        st.sync()
        if rc != 0:
            print(f"moe_decode failed: {rc}", file=sys.stderr)
            return 1
        flat = prof.cpu().numpy().astype(np.int64).reshape(T * L, PH, G)[L:]
        res = {}
        for a, b, name in PHASES:
            d = (flat[:, b, :] - flat[:, a, :]).astype(np.float64) / 1000.0
            res[name] = {"median_us": round(float(np.median(d)), 3),
                         "max_over_ctas_us": round(float(np.median(d.max(-1))), 3)}
        lay = (flat[1:, 0, :] - flat[:-1, 0, :]).astype(np.float64) / 1000.0
        print(json.dumps({"metric": "decode layer phases", "unit": "us",
                          "layer_us": round(float(np.median(lay)), 3), "phases": res,
                          "config": {"workload": f"{L} layers x {T} tokens, "
                                                 f"{'config-4' if args.c4 else 'config-1'} shapes",
                                     "early_copies": spec == 0, "grid": G, "data": "synthetic"}}), flush=True)
    st.close()
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--workload", default="config1",
                    choices=["config0", "config1", "config2", "config3", "config4", "layer", "phases",
                             "hostlink", "stream"])
    ap.add_argument("--attn-us", type=float, nargs="+", default=[0.0, 60.0],
                    help="stream: GPU time standing in for the rest of a layer, per layer")
    ap.add_argument("--c4", action="store_true", help="phases: config-4 shapes")
    ap.add_argument("--path", default="gemv", choices=["auto", "gemv", "gemm"])
    ap.add_argument("--c3-decode-steps", type=int, default=128)
    ap.add_argument("--c3-prefill-chunks", type=int, default=4)
    ap.add_argument("--no-ep", action="store_true",
                    help="headline: skip the expert-parallel (config 3) keys")
    ap.add_argument("--ep-decode-steps", type=int, default=32)
    ap.add_argument("--ep-prefill-chunks", type=int, default=2)
    ap.add_argument("--ep-exchange", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel dispatch/combine: peer-memory mailboxes or NCCL")
    ap.add_argument("--c2-warm", type=int, default=64)
    ap.add_argument("--c2-tokens", type=int, default=128)
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "config2":
        return run_config2(args)
    if args.workload == "config3":
        return run_config3(args)
    if args.workload == "config4":
        return run_config4(args)
    if args.workload == "layer":
        return run_layer(args)
    if args.workload == "phases":
        return run_phases(args)
    if args.workload == "hostlink":
        return run_hostlink(args)
    if args.workload == "config0":
        return run_config0(args)
    if args.workload == "stream":
        return run_stream(args)

    import torch
    import torch.distributed as dist
    from moe_prefetch_b200 import MoeStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    n_layers, tokens = args.layers, args.tokens
    st = MoeStack(n_layers=n_layers, device=local)
    st.synth_resident(seed=7919 * rank + 11)
    h = torch.from_numpy(ar1_states(tokens, N_EMBD, seed=12345 + rank)).cuda()
    out = torch.empty_like(h)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        st.decode(h, out)
    st.sync()

    props = torch.cuda.get_device_properties(local)
    bus = getattr(props, "pci_bus_id", None)
    bus = f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}" if isinstance(bus, int) else None
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(bus).start()
    time.sleep(0.3)
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    t_all0.record(stream)
    for i in range(args.steps):
        starts[i].record(stream)
        st.decode(h, out)
        ends[i].record(stream)
    t_all1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier()
    st.sync()
    total_ms = t_all0.elapsed_time(t_all1)
    launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    avg_launch_ms = sum(launch_ms) / len(launch_ms)
    t = torch.tensor([total_ms, avg_launch_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, avg_launch_ms = float(t[0]), float(t[1])
    value = world * args.steps * tokens / (total_ms / 1000.0)

    # end to end through the public API: pinned host in -> decode -> host out
    e2e = None
    if not args.no_e2e:
        hp = h.cpu().pin_memory()
        op = torch.empty_like(hp).pin_memory()
        for _ in range(max(1, args.warmup)):
            st.decode_host(hp, op)
        n_e2e = max(3, args.steps // 2)
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_e2e):
            st.decode_host(hp, op)
        e1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": world * n_e2e * tokens / (float(te[0]) / 1000.0), "unit": "tok/s",
               "h2d_bytes_per_step": tokens * N_EMBD * 4, "d2h_bytes_per_step": tokens * N_EMBD * 4,
               "steps": n_e2e}

    peak, peak_kind = measured_peaks()
    layer_token = LAYER_TOKEN_BYTES
    bytes_per_launch = layer_token * n_layers * tokens
    achieved = bytes_per_launch / (avg_launch_ms / 1000.0) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "k_decode_config1_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            tr = json.load(f)
        if tr.get("dram_bytes_per_layer_token"):
            traffic = float(tr["dram_bytes_per_layer_token"]) * n_layers * tokens
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "kernel": "moe::k_decode", "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": bytes_per_launch,
                "algorithmic_bytes_per_layer_token": layer_token}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_layers = []
        for il in range(2):
            g, u, d = st.slot_views(il)
            host_layers.append({"gate": g[:N_EXPERT].cpu().numpy(), "up": u[:N_EXPERT].cpu().numpy(),
                                "down": d[:N_EXPERT].cpu().numpy(),
                                "router": np.ascontiguousarray(
                                    np.random.default_rng(il).standard_normal((N_EXPERT, N_EMBD))
                                    .astype(np.float32) * np.float32(0.02))})
        threads = host_threads()
        v, n, el = cpu_baseline(host_layers, args.cpu_seconds, threads)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} layer-tokens over 2 host-resident layers in {el:.1f} s "
                         "(oracle's integer-dot CPU rows path, Q8_K activations, OpenMP); "
                         "tok/s = layer-tokens/s / 48"}

    # the expert-parallel workloads (config 3) on the same N GPUs, so that a
    # scaling run of this line carries their strong-scaling curve too; the
    # decode stack is freed first
    decode_geometry = st.decode_info()
    st.close()
    st = None
    ep = None
    if not args.no_ep:
        torch.cuda.empty_cache()
        ep_lines = ep_measure(world, rank, n_layers, args.ep_decode_steps, args.ep_prefill_chunks,
                              args.warmup, args.ep_exchange)
        ep = {}
        for ln in ep_lines:
            key = "decode" if "decode" in ln["metric"] else "prefill"
            ep[key] = {"value": ln["value"], "unit": "tok/s", "ms_per_step": ln["ms_per_step"],
                       "steps": ln["steps"], "workload": ln["config"]["workload"],
                       "path": ln["config"]["path"], "cuda_graph": ln["config"]["cuda_graph"],
                       "scaling": "strong"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded N(0,0.02) weights quantised on device; AR(1) inputs)",
            "config": config_block(tokens), "roofline": roofline, "cpu_baseline": cpu,
            "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
            "decode_geometry": decode_geometry,
            # config 3, expert-parallel over the same N GPUs (strong scaling)
            "expert_parallel": ep,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
