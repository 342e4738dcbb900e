"""The C ABI library loads without a GPU and exports every entry point that
include/moeb200.h declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moeb200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for must in ("moe_create", "moe_destroy", "moe_layer_forward", "moe_decode", "moe_step",
                 "moe_get_tables", "moe_get_stats", "moe_xc_prefetch", "moe_xc_query"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from moe_prefetch_b200 import _lib
    if not os.path.exists(_lib.LIB):
        pytest.fail("libmoeb200.so is not built (python -m moe_prefetch_b200.build)")
    lib = ctypes.CDLL(_lib.LIB)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes table covers the same surface
    assert set(_lib.SIGNATURES) == set(declared())


def test_bad_config_is_an_error_not_a_crash():
    from moe_prefetch_b200 import _lib
    lib = _lib.load()
    cfg = _lib.MoeCfg()
    cfg.n_layers = 1
    cfg.n_expert = 100             # not a multiple of 32
    cfg.n_used, cfg.n_embd, cfg.n_ff, cfg.down_type, cfg.n_slots = 8, 2048, 768, 14, 8
    out = ctypes.c_void_p()
    assert lib.moe_create(ctypes.byref(cfg), ctypes.byref(out)) == -4
    assert not out.value


def test_product_has_no_oracle_dependency():
    """The product package never imports the oracle (test infrastructure)."""
    pkg = os.path.join(ROOT, "moe_prefetch_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
                assert '#include "moe_oracle' not in src and "liboracle" not in src, f
