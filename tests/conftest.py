import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    return oracle.load()


@pytest.fixture(scope="session")
def emel():
    """The product package (directory emel.rs_b200), loaded under the module
    name emel_rs_b200."""
    from __graft_entry__ import load_package

    return load_package()
