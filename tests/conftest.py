import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(Path(__file__).resolve().parent) not in sys.path:
    sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) and the built libtessattn.so")


@pytest.fixture(scope="session")
def runtime():
    from tessery_b200 import CudaRuntime

    rt = CudaRuntime(0)
    yield rt
    rt.close()
