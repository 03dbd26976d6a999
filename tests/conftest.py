import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def pytest_sessionstart(session):
    # Rebuild the in-tree CUDA library (and the oracle) if any source is newer
    # than the built file; a no-op when they are up to date.
    from llmhost_b200 import build as kvbuild
    from oracle import oracle as O

    kvbuild.build()
    O.build()
