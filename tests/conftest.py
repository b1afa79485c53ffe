"""Shared test configuration.

Markers:
  gpu   needs a CUDA device (run on the B200 box: ``pytest -m gpu``); everything
        else runs on a CPU-only machine (``pytest -m "not gpu"``).
"""

import sys
from pathlib import Path

import pytest

TESTS = Path(__file__).resolve().parent
ROOT = TESTS.parent
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

# The reference package ``tokquay`` (installed next to the checkout by
# baseline/install_ref.sh): this library plugs into it, and the tests drive
# its own scheduler and engine.
import tokquay_b200._host  # noqa: E402,F401


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on the CPU")


@pytest.fixture(scope="session")
def golden():
    from helpers import load_golden

    return load_golden()


@pytest.fixture(scope="session")
def gpt2_weights():
    """float32 numpy weights of the random-init GPT-2 124M used by every config case."""
    from helpers import gpt2_small_weights

    return gpt2_small_weights()
