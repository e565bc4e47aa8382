import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) device")


def gpu_available():
    try:
        import fyodor_b200 as F
        return F.lib.fyb_device_count() > 0
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    # GPU tests are selected with -m gpu; they fail (not skip) without a device.
    pass


@pytest.fixture(scope="session")
def provider():
    import fyodor_b200 as F
    p = F.Provider()
    yield p
    p.close()
