import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "sr-hpm_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def ctx():
    import torch
    import srhpm_b200 as S
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    c = S.Context(0)
    yield c
    c.check()
    c.close()


@pytest.fixture(scope="session")
def ref():
    """The reference's own kernels compiled from its patch (None when the reference was absent at build time)."""
    import oracle as O
    return O.load_ref()
