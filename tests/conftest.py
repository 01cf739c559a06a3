import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cuda-triton-scala_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def gpu():
    """(Device, Stream, QuantizedGemmOps) on cuda:0 through libqgemm."""
    import qgemm
    dev = qgemm.Device(0)
    st = dev.stream()
    ops = qgemm.QuantizedGemmOps(st)
    yield dev, st, ops
    st.destroy()
    dev.close()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o
