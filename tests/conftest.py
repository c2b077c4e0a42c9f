import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.8-flash-next_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def built():
    """Builds libqmoe.so and the CPU checkers once per session."""
    import subprocess

    import oracle

    subprocess.run(["make", "-s", "-C", PKG], check=True)
    oracle.build()
    return True
