"""The ExpertCache fixture is the reference's own output: regenerated here from
the reference tree (src/prefetch_engine.py, run on the host by
tests/golden/make_golden.py) it must equal the committed file.  The GPU test
(test_gpu_expert_cache.py) replays it through the C ABI."""
import json
import os

import pytest

from conftest import REFERENCE

HERE = os.path.dirname(os.path.abspath(__file__))


def test_expert_cache_fixture_is_the_references_output():
    if not os.path.exists(os.path.join(REFERENCE, "src", "prefetch_engine.py")):
        pytest.skip("reference tree not present")
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with open(os.path.join(HERE, "golden", "expert_cache.json")) as f:
        committed = json.load(f)
    assert mod.expert_cache_cases() == committed
