"""pytest configuration: the `gpu` marker, import paths, shared fixtures.

`-m "not gpu"` runs here without a GPU: the oracle against the golden fixtures (and against the
reference's own library where it was built), the host logic and the C-ABI symbol table.
`-m gpu` runs the parity tests proper: CUDA results through the C ABI against the oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "tesseract-npu_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (parity tests through the C ABI)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def tsro():
    import oracle
    oracle.build(ref=True)
    return oracle.Tsro()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.Ref.available():
        pytest.skip("the reference library (oracle/_ref) was not built on this machine")
    return oracle.Ref()


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tsrc
    d = tsrc.Device(0)
    yield d
    d.close()
