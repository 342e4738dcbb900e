import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REFERENCE = "/root/reference"

# Output tolerances of north_star, against the fp32-accumulated oracle
REL_L2_TOL = 1e-3
MAX_ABS_TOL = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def rms_norm(h, eps=0.0):
    h = np.asarray(h, np.float32)
    return (h / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)).astype(np.float32)


def ar1_states(n_tok, n_embd, rho=0.9, seed=12345):
    """AR(1) hidden states h_t = rho h_{t-1} + sqrt(1-rho^2) eps_t, RMS-normed."""
    rng = np.random.default_rng(seed)
    h = np.empty((n_tok, n_embd), np.float32)
    prev = rng.standard_normal(n_embd)
    for t in range(n_tok):
        prev = rho * prev + np.sqrt(1 - rho * rho) * rng.standard_normal(n_embd)
        h[t] = prev
    return rms_norm(h)
