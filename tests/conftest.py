import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (runs the sm_100a kernels)")
    config.addinivalue_line("markers", "slow: long CPU oracle runs (still part of the default CPU suite)")


@pytest.fixture(scope="session")
def M():
    from streaming_machine_b200 import convert
    return convert.load_gpt2(0)


@pytest.fixture(scope="session")
def orc(M):
    from oracle.oracle import Oracle
    return Oracle(M)


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(GOLDEN, "gpt2_seed0.json")) as f:
        return json.load(f)


def gload(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def PM():
    """The seeded Pythia-160M machine (keys of the reference converter's base2_pythia-160m.npz)."""
    from streaming_machine_b200 import convert
    return convert.load_pythia(0)


@pytest.fixture(scope="session")
def porc(PM):
    from oracle.oracle import PythiaOracle
    return PythiaOracle(PM)


@pytest.fixture(scope="session")
def pgold():
    import json
    with open(os.path.join(GOLDEN, "pythia_seed0.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def gpu_engine(M):
    """One engine per session (uploading the weights and building their layouts is the costly part)."""
    from streaming_machine_b200 import engine
    e = engine.Engine(M, n_streams=1, max_ctx=64)
    yield e
    e.close()


@pytest.fixture(scope="session")
def pythia_engine(PM):
    from streaming_machine_b200 import engine
    e = engine.Engine(PM, n_streams=1, max_ctx=128)
    yield e
    e.close()


def with_streams(e, n_streams, max_ctx):
    """Re-shape the engine's stream slots only when needed."""
    if (e.n_streams, e.max_ctx) != (n_streams, max_ctx):
        e.alloc_streams(n_streams, max_ctx)
    return e
