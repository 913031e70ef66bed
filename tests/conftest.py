"""Shared test set-up: the gpu marker, import paths for the package
(smollm2.c_b200/ is not an importable package name) and the oracle."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "smollm2.c_b200"), os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA library)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    return orc.Oracle()


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(REPO, "tests", "golden", "golden.json")) as f:
        return json.load(f)
