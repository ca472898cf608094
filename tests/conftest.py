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


# Near-tie census of the routing parity tests: name -> {tokens, near_ties,
# near_ties_differing}.  Printed at the end of the run (also under -q).
NEAR_TIES = {}


def record_near_ties(name, tokens, near, near_diff):
    NEAR_TIES[name] = {"tokens": int(tokens), "near_ties": int(near), "near_ties_differing": int(near_diff)}


def pytest_terminal_summary(terminalreporter):
    if not NEAR_TIES:
        return
    tr = terminalreporter
    tr.section("routing near ties (oracle top-(K+1) logit margin < 1e-3)")
    for name in sorted(NEAR_TIES):
        v = NEAR_TIES[name]
        tr.write_line(f"{name}: {v['near_ties']} of {v['tokens']} tokens are near ties, "
                      f"{v['near_ties_differing']} of those differ from the oracle")
    out = os.environ.get("MOE_NEAR_TIES_JSON")
    if out:
        import json

        with open(out, "w") as f:
            json.dump(NEAR_TIES, f, indent=1, sort_keys=True)
