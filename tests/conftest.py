import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "late: collected after every other test")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


def pytest_collection_modifyitems(config, items):
    """Tests marked ``late`` run after all others (stable order otherwise), so a
    run that stops at its first failure has run every other test already."""
    items[:] = [it for it in items if it.get_closest_marker("late") is None] + \
               [it for it in items if it.get_closest_marker("late") is not None]
