import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_package():
    """Loads audio.cpp_b200/ (a directory whose name is not an identifier) as module audiocpp_b200."""
    if "audiocpp_b200" in sys.modules:
        return sys.modules["audiocpp_b200"]
    path = os.path.join(ROOT, "audio.cpp_b200", "__init__.py")
    spec = importlib.util.spec_from_file_location("audiocpp_b200", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["audiocpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def b2d():
    return load_package()


@pytest.fixture(scope="session")
def ctx(b2d):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    c = b2d.Context(0)
    yield c
    c.close()
