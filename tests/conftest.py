import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture
def scratch(request):
    """A fresh directory for one test's files inside the repository
    (tests/_scratch/<test>), removed afterwards."""
    import re
    import shutil
    d = ROOT / "tests" / "_scratch" / re.sub(r"[^A-Za-z0-9_.-]", "_", request.node.name)
    shutil.rmtree(d, ignore_errors=True)
    d.mkdir(parents=True)
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture(scope="session")
def native():
    """The C-ABI library (built if missing)."""
    from swarmlora_b200 import build, _native
    if not _native.LIB_PATH.exists():
        build.build()
    return _native


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    return torch.device("cuda:0")
