import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native extension")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def _fresh_managers():
    yield
    from flextensor_b200.runtime import manager as m

    for om in list(m._registry.values()):
        try:
            om.release()
        except Exception:  # noqa: BLE001
            pass
    m._registry.clear()
