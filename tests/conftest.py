import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle"))
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__ as ge
    ge.build(force=False)   # compiles only what is older than its sources
    return ge.load_package()


@pytest.fixture(scope="session")
def oracle():
    import __graft_entry__ as ge
    ge._load_file("hy_oracle_build", os.path.join(REPO, "oracle", "build.py")).build()
    import hy_oracle
    return hy_oracle


def load_golden(name):
    import numpy as np
    path = os.path.join(GOLDEN, f"{name}.npz")
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name} not generated")
    return dict(np.load(path))
