"""The just-in-time streaming planner (moe_prefetch_b200/csrc/moe_planner.h)
against the reference's own unit test of its planner, cpp/test-moe-planner.cpp
(dedupe and deadline refresh, earliest-deadline-first order, chunking, late
and posted drops, hold, preemption at chunk boundaries, reset).  oracle/Makefile
compiles that test, where it lies in the reference tree, against this
project's header; it must print PASS."""
import os
import subprocess

import pytest

from conftest import REFERENCE, ROOT


def test_reference_planner_test_passes_on_our_planner():
    src = os.path.join(REFERENCE, "cpp", "test-moe-planner.cpp")
    if not os.path.exists(src):
        pytest.skip("reference tree not present")
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle"),
                           os.path.join(ROOT, "oracle", "_ref", "test-moe-planner"), "REF=" + REFERENCE])
    r = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "test-moe-planner")], capture_output=True,
                       text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("PASS: planner"), r.stdout
