import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libgollama_cuda.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")
    config.addinivalue_line(
        "markers",
        "unvalidated: a GPU test of an opt-in kernel variant that has not yet passed on a B200; "
        "skipped unless GLC_RUN_UNVALIDATED=1",
    )


def pytest_collection_modifyitems(config, items):
    if os.environ.get("GLC_RUN_UNVALIDATED") == "1":
        return
    skip = pytest.mark.skip(reason="opt-in variant not yet run on a B200 (set GLC_RUN_UNVALIDATED=1)")
    for item in items:
        if "unvalidated" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ctx():
    from gollama_b200.device import Context

    c = Context(int(os.environ.get("GLC_TEST_DEVICE", "0")))
    yield c
    c.close()
