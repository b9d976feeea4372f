"""pytest configuration: the `gpu` marker and shared fixtures.

GPU tests (marked `gpu`) call the product library through its C ABI and
compare against the CPU oracle (oracle/); they need a B200.  Everything else
runs on a CPU-only host.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle.oracle import RefLib, ref_library_path
    if not os.path.exists(ref_library_path()):
        pytest.skip("oracle/_ref not built (needs the reference sources at build time)")
    return RefLib()


@pytest.fixture(scope="session")
def ctx():
    import mfft_bench_b200 as m
    if m.device_count() < 1:
        pytest.fail("GPU test run without a visible CUDA device")
    c = m.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


def load_fixture(name):
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", name))
