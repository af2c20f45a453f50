import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def fixtures():
    import json
    return json.loads((ROOT / "tests/golden/reference_fixtures.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    """The native library on a real GPU; the product has no fallback, so a missing library
    or device is a failure of every gpu test, not a skip."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from peregrine_b200 import build, capi
    build.build()
    capi.lib()
    return capi
