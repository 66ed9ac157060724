import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "threedgaussiansplatting.jl_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA path")


@pytest.fixture(scope="session")
def golden():
    import json
    return json.loads((REPO / "tests" / "golden" / "reference_golden.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    """The CUDA library on cuda:0; fails loudly when the extension is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import gs3d
    gs3d.lib()
    return torch.device("cuda:0")
