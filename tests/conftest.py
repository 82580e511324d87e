import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")
    config.addinivalue_line("markers", "multigpu: needs >= 2 CUDA devices")
    config.addinivalue_line("markers", "slow: full-size case (minutes on CPU)")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build(ref=Path(os.environ.get("AMP_REF", "/root/reference")).exists())
    return oracle


@pytest.fixture(scope="session")
def amp_lib():
    """libamp_b200.so, built in-tree if it is missing (nvcc cross-compiles on CPU)."""
    import amp_b200
    from amp_b200 import build
    if not amp_b200.LIB_PATH.exists():
        build.build()
    return amp_b200.lib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
    return torch.device("cuda:0")
