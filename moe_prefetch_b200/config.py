"""Configuration of the slot cache, with the reference's switch names.

The reference reads ``--moe-expert-cache N`` / ``--moe-expert-cache-inserts K``
from the llama.cpp command line and a set of ``LLAMA_MOE_*`` environment
variables in llama_moe_cache_init (patches/0006:501-520, 0007:492-506,
0008:536-573).  ``MoeCacheConfig.from_env`` parses the same names with the
same meaning and the same defaults, so a deployment's switches carry over.
"""
import dataclasses
import os
import sys

ADMIT_MODES = {"off": 0, "0": 0, "": 0, "heat": 1, "window": 2}


@dataclasses.dataclass
class MoeCacheConfig:
    n_slots: int = 0               # --moe-expert-cache N (0 = every expert resident)
    max_inserts: int = 2           # --moe-expert-cache-inserts K (patches/0006:161)
    slot_profile: str = ""         # LLAMA_MOE_SLOT_PROFILE "il:n,il:n,..."
    admit: str = "off"             # LLAMA_MOE_ADMIT off | heat | window
    admit_window: int = 8          # LLAMA_MOE_ADMIT_WINDOW
    admit_half: int = 64           # LLAMA_MOE_ADMIT_HALF
    admit_floor: float = 1.0       # LLAMA_MOE_ADMIT_FLOOR
    spec_probation: bool = False   # LLAMA_MOE_SPEC_PROBATION
    batch_tables: bool = False     # LLAMA_MOE_BATCH_TABLES
    cache_prior: float = 0.0       # LLAMA_MOE_CACHE_PRIOR (delta)
    heat_file: str = ""            # LLAMA_MOE_HEAT_FILE
    early_issue: bool = False      # LLAMA_MOE_EARLY_ISSUE
    predict_top: int = 3           # LLAMA_MOE_PREDICT_TOP
    evictor: str = ""              # LLAMA_MOE_EVICTOR (MOEP v3 file)
    stream: bool = False           # LLAMA_MOE_STREAM (just-in-time streaming; needs early_issue)
    stream_per_layer: int = 4      # LLAMA_MOE_STREAM_PER_LAYER
    stream_reserve: int = 2        # LLAMA_MOE_STREAM_RESERVE
    stream_gbps: float = 45.7      # LLAMA_MOE_STREAM_GBPS
    stream_topk: int = 8           # LLAMA_MOE_STREAM_TOPK
    freeze: bool = False           # LLAMA_MOE_CACHE_FREEZE
    deterministic: bool = True     # LLAMA_MOE_DETERMINISTIC (always on here)
    map_record: str = ""           # LLAMA_MOE_MAP_RECORD
    map_replay: str = ""           # LLAMA_MOE_MAP_REPLAY
    route_trace: str = ""          # LLAMA_MOE_ROUTE_TRACE

    @property
    def admit_mode(self):
        return ADMIT_MODES.get(self.admit, 0)

    @classmethod
    def from_env(cls, env=None, argv=None):
        """Parse LLAMA_MOE_* from `env` (default os.environ) and the two CLI
        flags from `argv`, with the reference's rules: unknown LLAMA_MOE_ADMIT
        values warn and admit every miss; ADMIT_HALF / ADMIT_WINDOW are clamped
        to >= 1; CACHE_PRIOR to >= 0 (patches/0007:492-506)."""
        env = os.environ if env is None else env
        c = cls()
        argv = list(argv or [])
        for i, a in enumerate(argv):
            if a == "--moe-expert-cache" and i + 1 < len(argv):
                c.n_slots = int(argv[i + 1])
            elif a == "--moe-expert-cache-inserts" and i + 1 < len(argv):
                v = int(argv[i + 1])
                if v > 0:
                    c.max_inserts = v

        def get(name):
            return env.get(name)

        if get("LLAMA_MOE_SLOT_PROFILE") is not None:
            c.slot_profile = get("LLAMA_MOE_SLOT_PROFILE")
        a = get("LLAMA_MOE_ADMIT")
        if a is not None:
            if a in ADMIT_MODES:
                c.admit = a if a in ("heat", "window") else "off"
            else:
                print(f"moe-cache: LLAMA_MOE_ADMIT='{a}' NOT UNDERSTOOD (heat | window | off)"
                      " - admitting every miss", file=sys.stderr)
                c.admit = "off"
        if get("LLAMA_MOE_ADMIT_HALF") is not None:
            c.admit_half = max(1, _atoi(get("LLAMA_MOE_ADMIT_HALF")))
        if get("LLAMA_MOE_ADMIT_FLOOR") is not None:
            c.admit_floor = _atof(get("LLAMA_MOE_ADMIT_FLOOR"))
        if get("LLAMA_MOE_ADMIT_WINDOW") is not None:
            c.admit_window = max(1, _atoi(get("LLAMA_MOE_ADMIT_WINDOW")))
        for name, attr in (("LLAMA_MOE_SPEC_PROBATION", "spec_probation"),
                           ("LLAMA_MOE_BATCH_TABLES", "batch_tables"),
                           ("LLAMA_MOE_EARLY_ISSUE", "early_issue"),
                           ("LLAMA_MOE_CACHE_FREEZE", "freeze"),
                           ("LLAMA_MOE_DETERMINISTIC", "deterministic")):
            if get(name) is not None:
                setattr(c, attr, _atoi(get(name)) != 0)
        if get("LLAMA_MOE_CACHE_PRIOR") is not None:
            c.cache_prior = max(0.0, _atof(get("LLAMA_MOE_CACHE_PRIOR")))
        if get("LLAMA_MOE_PREDICT_TOP") is not None:
            c.predict_top = _atoi(get("LLAMA_MOE_PREDICT_TOP"))
        # streaming switches (patches/0010:1828-1832, 1963): per_layer >= 1,
        # reserve >= 0, GB/s >= 1, topk in [1, 8]
        if get("LLAMA_MOE_STREAM") is not None:
            c.stream = _atoi(get("LLAMA_MOE_STREAM")) != 0
        if get("LLAMA_MOE_STREAM_PER_LAYER") is not None:
            c.stream_per_layer = max(1, _atoi(get("LLAMA_MOE_STREAM_PER_LAYER")))
        if get("LLAMA_MOE_STREAM_RESERVE") is not None:
            c.stream_reserve = max(0, _atoi(get("LLAMA_MOE_STREAM_RESERVE")))
        if get("LLAMA_MOE_STREAM_GBPS") is not None:
            c.stream_gbps = max(1.0, _atof(get("LLAMA_MOE_STREAM_GBPS")))
        if get("LLAMA_MOE_STREAM_TOPK") is not None:
            c.stream_topk = min(8, max(1, _atoi(get("LLAMA_MOE_STREAM_TOPK"))))
        for name, attr in (("LLAMA_MOE_HEAT_FILE", "heat_file"),
                           ("LLAMA_MOE_EVICTOR", "evictor"),
                           ("LLAMA_MOE_MAP_RECORD", "map_record"),
                           ("LLAMA_MOE_MAP_REPLAY", "map_replay"),
                           ("LLAMA_MOE_ROUTE_TRACE", "route_trace")):
            if get(name) is not None:
                setattr(c, attr, get(name))
        if c.freeze:
            c.max_inserts = 0
        if c.map_replay:
            c.freeze = True
            c.max_inserts = 0
        return c

    def slots_per_layer(self, n_layers, n_expert):
        """Per-layer slot counts: the profile's overrides, else n_slots (0 ->
        every expert resident)."""
        dflt = self.n_slots if self.n_slots > 0 else n_expert
        prof = parse_slot_profile(self.slot_profile)
        return [prof.get(il, dflt) for il in range(n_layers)]


def _atoi(s):
    """C atoi: leading integer, 0 if none."""
    s = s.strip()
    n, i = 0, 0
    sign = 1
    if i < len(s) and s[i] in "+-":
        sign = -1 if s[i] == "-" else 1
        i += 1
    while i < len(s) and s[i].isdigit():
        n = n * 10 + int(s[i])
        i += 1
    return sign * n


def _atof(s):
    s = s.strip()
    for j in range(len(s), 0, -1):
        try:
            return float(s[:j])
        except ValueError:
            continue
    return 0.0


def parse_slot_profile(spec):
    """"il:slots,il:slots,..." -> {il: slots}; stops at the first malformed
    entry and ignores counts <= 0 by stopping (load_slot_profile,
    patches/0006:461-480)."""
    out = {}
    if not spec:
        return out

    def scan_int(s, i):
        # sscanf "%d": optional whitespace, optional sign, at least one digit
        while i < len(s) and s[i] in " \t\n\r\f\v":
            i += 1
        j = i
        if j < len(s) and s[j] in "+-":
            j += 1
        k = j
        while k < len(s) and s[k].isdigit():
            k += 1
        if k == j:
            return None, i
        return int(s[i:k]), k

    p = 0
    while p < len(spec):
        il, q = scan_int(spec, p)
        if il is None or q >= len(spec) or spec[q] != ":":
            break
        n, q = scan_int(spec, q + 1)
        if n is None or n <= 0:
            break
        out[il] = n
        p = q
        if p < len(spec) and spec[p] == ",":
            p += 1
        else:
            break
    return out


def format_slot_profile(caps):
    return ",".join(f"{il}:{n}" for il, n in enumerate(caps))


def greedy_allocate_bytes(per_layer_miss8, grid, n_layers, uniform_cap, frozen_layers,
                          expert_bytes):
    """Byte-priced greedy slot allocation, the reference's
    experiments/p7_slot_allocation.py:144-185 (greedy_allocate_bytes).

    Each layer starts at the bottom of `grid` (frozen layers sit at
    uniform_cap and never move).  The byte budget is what uniform_cap slots in
    every layer would take.  A move lifts one layer to its next grid size; its
    value is the drop in that layer's misses (per_layer_miss8[slots][layer])
    per byte it costs.  The most valuable move is made while it fits in what
    is left of the budget (ties: lower layer first); a move that does not fit
    is dropped for good, as in the reference.  A layer with no recorded
    expert size is priced at the mean of the known sizes.
    Returns (caps, bytes used, budget)."""
    sized = [b for b in expert_bytes if b]
    fallback = sum(sized) / len(sized)
    price = [b if b else fallback for b in expert_bytes]        # bytes per slot
    budget = sum(uniform_cap * price[il] for il in range(n_layers))
    pinned = set(frozen_layers)
    level = [0] * n_layers                                       # grid position
    caps = [uniform_cap if il in pinned else grid[0] for il in range(n_layers)]
    left = budget - sum(caps[il] * price[il] for il in range(n_layers))

    def next_move(il):
        """(misses saved per byte, bytes) of lifting layer il one grid step,
        or None at the top of the grid or for a frozen layer."""
        if il in pinned or level[il] + 1 >= len(grid):
            return None
        lo, hi = grid[level[il]], grid[level[il] + 1]
        nbytes = (hi - lo) * price[il]
        return (per_layer_miss8[lo][il] - per_layer_miss8[hi][il]) / nbytes, nbytes

    open_moves = {}                                              # layer -> value
    for il in range(n_layers):
        mv = next_move(il)
        if mv is not None and mv[0] > 0:
            open_moves[il] = mv[0]
    while open_moves:
        il = max(open_moves, key=lambda q: (open_moves[q], -q))
        del open_moves[il]
        _, nbytes = next_move(il)
        if nbytes > left:
            continue
        level[il] += 1
        caps[il] = grid[level[il]]
        left -= nbytes
        mv = next_move(il)
        if mv is not None and mv[0] > 0:
            open_moves[il] = mv[0]
    used = sum(caps[il] * price[il] for il in range(n_layers))
    return caps, used, budget
