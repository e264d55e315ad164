import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def ncz():
    import importlib

    return importlib.import_module("not-cute-zig_b200")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    return oracle


@pytest.fixture
def fake(ncz):
    """The library's driver-call table swapped for eight fake devices
    (tests/fake_driver.py) for one test; on the way out the CUDA runtime is
    restored and nothing the library made may be left alive."""
    from tests import fake_driver

    f = fake_driver.FakeDevices(8)
    assert ncz.driver.install(f.table()) == 0
    yield f
    ncz.driver.install(None)
    assert f.live() == {"streams": 0, "events": 0, "pools": 0, "allocs": 0}
    assert f.errors == []
