import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "bitmask-speculation_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    return json.loads((GOLDEN / "golden.json").read_text())


@pytest.fixture(scope="session")
def cuda_module():
    """The native module; on a machine with a GPU a missing build is a failure."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("NVIDIA CUDA device required")
    from bitmask_speculation_b200.kernels._extension import load_extension
    return load_extension()
