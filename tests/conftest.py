"""Test configuration: the `gpu` marker, import paths, and shared fixtures.

`-m "not gpu"` runs the oracle against the reference's own known-answer vectors, the host-side
logic and the C-ABI surface (no compute without a GPU); `-m gpu` runs the parity tests proper,
which call the CUDA library through its C ABI and compare with the oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tsfm-zig_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls the library through its C ABI")


@pytest.fixture(scope="session")
def kat():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "kat.json")) as f:
        return json.load(f)


