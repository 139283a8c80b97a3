import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests run only where a GPU exists; without one they fail loudly."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    from ffn_residual_mesh_b200 import build
    build.build()
    return torch.device("cuda:0")
