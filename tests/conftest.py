"""pytest configuration: import paths, the `gpu` marker, and the reference's
correctness-warnings fixture (tests/conftest.py of the reference turns
RL_TRITON_CORRECTNESS_WARNINGS on for every non-perf test)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "rl-triton_b200"), ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA path through the C ABI")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(autouse=True)
def set_correctness_warnings(request):
    old = os.environ.get("RL_TRITON_CORRECTNESS_WARNINGS")
    os.environ["RL_TRITON_CORRECTNESS_WARNINGS"] = "1"
    yield
    if old is None:
        del os.environ["RL_TRITON_CORRECTNESS_WARNINGS"]
    else:
        os.environ["RL_TRITON_CORRECTNESS_WARNINGS"] = old
