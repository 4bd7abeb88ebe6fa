import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs through libnsq's C ABI)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "dequant_golden.npz")))


@pytest.fixture
def tuning(monkeypatch):
    """Sets NSQ_* launch-planning variables for one test.  libnsq reads them
    once, so every change is followed by nsq_reload_tuning; afterwards the
    previous environment is restored and read again."""
    from planejaja_b200 import _lib
    lib = _lib.load()

    class Tuning:
        def set(self, name, value):
            monkeypatch.setenv(name, str(value))
            lib.nsq_reload_tuning()

        def unset(self, name):
            monkeypatch.delenv(name, raising=False)
            lib.nsq_reload_tuning()

    yield Tuning()
    monkeypatch.undo()
    lib.nsq_reload_tuning()
