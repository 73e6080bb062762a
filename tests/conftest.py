import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


@pytest.fixture(scope="session")
def cuda_ctx():
    """The library context on cuda:0. GPU tests never skip silently: a missing
    GPU or library is an error."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from molten_b200 import build
    build.build()
    from molten_b200 import lfm
    ctx = lfm.Context(0)
    yield ctx
    ctx.close()
