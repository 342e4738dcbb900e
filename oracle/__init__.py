"""CPU oracle for the MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this package, and only as the checker (or as the timed CPU baseline).
The product path in ``moe_prefetch_b200`` never imports it.
"""
from .oracle import *  # noqa: F401,F403
