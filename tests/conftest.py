import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA path against the oracle")


@pytest.fixture(scope="session")
def dllm():
    return importlib.import_module("distributed-llm1_b200")


@pytest.fixture(scope="session")
def weights_cache():
    return {}


@pytest.fixture(autouse=True)
def _release_device_objects():
    """Contexts, stages and buffers hold device memory; free them between tests."""
    yield
    import gc
    gc.collect()
