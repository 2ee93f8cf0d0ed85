import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "llama3-java-hat_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(ROOT, "tests", "golden", "known_answers.json")) as f:
        return {c["id"]: c for c in json.load(f)["cases"]}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def acc():
    import llamahat
    return llamahat.Accelerator(0)


@pytest.fixture(scope="session")
def tiny_weights():
    from llamahat.config import TINY
    from llamahat.synth import synth_weights
    return TINY, synth_weights(TINY, seed=7)
