"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on the CPU."""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mocha-moze-llm_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)

import mocha_q8  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def golden_q8():
    with open(os.path.join(ROOT, "tests", "golden", "q8_golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def q8_model_path(golden_q8):
    return mocha_q8.model_path(golden_q8["model_seed"])


@pytest.fixture(scope="session")
def q8_model_bytes(q8_model_path):
    return np.fromfile(q8_model_path, dtype=np.uint8)


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle_py
    oracle_py.build(ref=False)
    return oracle_py


@pytest.fixture(scope="session")
def native():
    import mocha_native
    if not os.path.exists(mocha_native.LIB_PATH):
        mocha_native.build()
    return mocha_native
