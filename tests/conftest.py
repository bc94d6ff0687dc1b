"""Shared test set-up.

Markers: ``gpu`` tests need a CUDA device (a B200) and call the product
through its C ABI; everything else runs on a CPU-only machine.
"""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers",
                            "gpu: needs a CUDA GPU; calls the CUDA library")


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name))


def unpack(d, key, i):
    off, ln = d[key + "_off"][i], d[key + "_len"][i]
    return d[key + "_data" if key + "_data" in d else key][off:off + ln]


def scenarios():
    with open(os.path.join(GOLDEN, "store_scenarios.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def sha_cases():
    return load_npz("sha256_cases.npz")


@pytest.fixture(scope="session")
def kvq8_cases():
    return load_npz("kvq8_cases.npz")
