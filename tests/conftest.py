import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")
if GOLDEN not in sys.path:  # the fixture generators also define how some inputs are regenerated
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    """``{case: {key: array}}`` from one of the reference-generated fixture files."""
    data = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    cases: dict = {}
    for key in data.files:
        case, _, rest = key.partition("/")
        cases.setdefault(case, {})[rest] = data[key]
    return cases


@pytest.fixture(scope="session")
def golden_single():
    return load_golden("attention_single.npz")


@pytest.fixture(scope="session")
def golden_sp():
    return load_golden("sequence_parallel.npz")


@pytest.fixture(scope="session")
def golden_cache():
    return load_golden("kv_cache.npz")


@pytest.fixture(scope="session")
def golden_cache_engine():
    import json

    with open(os.path.join(GOLDEN, "kv_cache_engine.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_wire():
    return load_golden("ring_wire.npz")


@pytest.fixture(scope="session")
def golden_llama():
    data = np.load(os.path.join(GOLDEN, "llama_sp.npz"), allow_pickle=False)
    return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def golden_config1():
    data = np.load(os.path.join(GOLDEN, "config1.npz"), allow_pickle=False)
    return {k: data[k] for k in data.files}
