import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The reference's operator tolerance: |a - b| <= 1e-5 + 1e-4 |b|
# (tests/basic_ops.rs:8-9, tests/model.rs:19).
ATOL, RTOL = 1e-5, 1e-4


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


def golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def assert_close(actual, expected, atol=ATOL, rtol=RTOL, name=""):
    a = np.asarray(actual, dtype=np.float64).ravel()
    b = np.asarray(np.asarray(expected, dtype=np.float32), dtype=np.float64).ravel()
    assert a.shape == b.shape, (name, a.shape, b.shape)
    assert np.all(np.isfinite(a)), name
    err = np.abs(a - b)
    budget = atol + rtol * np.abs(b)
    bad = np.nonzero(err > budget)[0]
    assert bad.size == 0, f"{name}: {bad.size} over budget, first {bad[0]}: {a[bad[0]]} vs {b[bad[0]]}"


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture
def oracle(oracle_lib):
    # Interleaved evaluation: bit-identical to the one-row-at-a-time loop
    # (tests/test_oracle.py::test_interleaved_and_chunked_paths_bit_identical)
    # and several times faster for the model-sized parity tests.
    oracle_lib.set_fast(True)
    return oracle_lib
