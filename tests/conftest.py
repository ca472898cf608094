import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def moe():
    from _moe_loader import load

    return load()


@pytest.fixture(scope="session")
def O():
    """The CPU checkers (oracle/): built on first use if the prebuilt .so is absent."""
    from oracle import oracle

    if not os.path.isfile(oracle.ORACLE_SO):
        oracle.build(None)
    return oracle


GOLDEN_DIR = os.path.join(HERE, "golden")


def golden_cases():
    return sorted(f[:-4] for f in os.listdir(GOLDEN_DIR) if f.endswith(".npz"))
