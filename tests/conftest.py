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


# late test files, in the order they run (the hot path's next rows first); late files not listed run after
LATE_ORDER = ("test_recovery_walk_gpu", "test_linear_argmax_gpu", "test_wait_timeouts_gpu", "test_peer_gpu",
              "test_draft_gpu")


def _module(item) -> str:
    return os.path.splitext(os.path.basename(str(item.fspath)))[0]


def pytest_collection_modifyitems(config, items):
    """Tests marked ``late`` run after all others (stable order otherwise), so a
    run that stops at its first failure has run every other test already;
    among them LATE_ORDER decides.  Files named ``test_zz_*`` run last of all."""
    def key(it):
        mod = _module(it)
        if mod.startswith("test_zz_"):
            return (2, 0)
        if it.get_closest_marker("late") is None:
            return (0, 0)
        return (1, LATE_ORDER.index(mod) if mod in LATE_ORDER else len(LATE_ORDER))

    items[:] = sorted(items, key=key)  # stable: the collection order within each group
