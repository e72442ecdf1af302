import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer-running parity case")


@pytest.fixture(scope="session")
def model_cache(tmp_path_factory):
    d = os.environ.get("C2S_MODEL_CACHE")
    if not d:
        d = str(tmp_path_factory.mktemp("models"))
        os.environ["C2S_MODEL_CACHE"] = d
    return d
