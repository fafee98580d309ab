"""pytest configuration: the `gpu` marker, and in-tree builds of the library
and of the test oracle before any test runs (both are cheap when up to date)."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session", autouse=True)
def _built():
    from libcusort_b200 import build as b
    b.build()
    from oracle import oracle as o
    if not o.ORACLE_SO.exists():
        o.build(ref=False)
    yield
