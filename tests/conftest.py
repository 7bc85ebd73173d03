import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def accept_golden():
    return load_golden("accept.json")


@pytest.fixture(scope="session")
def reorder_golden():
    return load_golden("reorder.json")


@pytest.fixture(scope="session")
def mask_golden():
    return load_golden("mask.json")
