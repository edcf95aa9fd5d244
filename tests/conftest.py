"""pytest configuration: the `gpu` marker and import paths.

`python -m pytest tests -m "not gpu"` runs on any machine (oracle vs golden fixtures, host logic,
the C-ABI symbol table, gloo ranks); `-m gpu` needs an sm_100 GPU and runs the parity tests
proper through the C ABI.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
