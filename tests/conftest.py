import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    # Build the checker (oracle) and the product library if a source changed; both are cheap.
    import oracle
    oracle.build()
    from flour_b200 import build as fb
    if fb.needs_build():
        fb.build()


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def device():
    import torch
    return torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
