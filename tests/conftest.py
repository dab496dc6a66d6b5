import os
import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the host libraries the tests need (cheap when up to date)."""
    from dpuf_b200 import _native
    from oracle import oracle as orc

    _native.build_pack()
    orc.build()
    yield


@pytest.fixture
def env_knobs():
    """Set reference environment knobs for one test and restore them afterwards."""
    saved = {}

    def set_(pairs):
        for k, v in pairs:
            saved.setdefault(k, os.environ.get(k))
            os.environ[k] = v

    yield set_
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
