import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def orc():
    import oracle
    if not os.path.exists(oracle.LIB_PATH):
        oracle.build()
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def api():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from nvfp4bench_b200 import api as _api
    _api.lib()
    return _api
