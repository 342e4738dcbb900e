"""moe_prefetch_b200 -- a B200-native MoE layer with a GPU expert slot cache.

The hot path of a Q4_K_M Qwen3-A3B-class MoE layer behind the operator API of
everett6/moe-prefetch's ``--moe-expert-cache`` (per-layer slots, second-miss
admission, byte-priced slot profiles, batched table writes, cache-prior routing
delta) and its ``ExpertCache`` / predictor hook.  Python host code drives a thin
C ABI (include/moeb200.h, libmoeb200.so) of hand-written sm_100a kernels.
"""
from .config import (MoeCacheConfig, format_slot_profile, greedy_allocate_bytes,  # noqa: F401
                     parse_slot_profile)
from ._lib import QTYPE_Q4_K, QTYPE_Q6_K, MoeError  # noqa: F401


def __getattr__(name):
    # torch-dependent pieces load lazily, so the config helpers import without CUDA
    if name in ("MoeStack", "expert_bytes", "load_heat", "save_heat"):
        from . import stack
        return getattr(stack, name)
    if name in ("ExpertCache", "EXPERT_BYTES", "EXPERT_MIB"):
        from . import prefetch_engine
        return getattr(prefetch_engine, name)
    if name in ("MoePredictor", "ExpertPredictor"):
        from . import predictor
        return getattr(predictor, name)
    raise AttributeError(name)
