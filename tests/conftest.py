import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    """The package with libtla.so built (make is a no-op when up to date)."""
    import __graft_entry__ as ge

    subprocess.run(["make", "-s", "-j8", "-C", str(ROOT / "three-llm_b200" / "csrc")], check=True)
    return ge.load_package()


@pytest.fixture(scope="session")
def cuda(pkg):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
