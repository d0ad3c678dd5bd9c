import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU-side checks")


def pytest_collection_modifyitems(config, items):
    # GPU tests are selected with -m gpu; without a device they are skipped
    # rather than silently run on something else.
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def gxlib():
    from galactus_b200 import build as b
    b.build()
    import galactus_b200
    return galactus_b200


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.build()
    o.lib()
    return o


@pytest.fixture(scope="session")
def dev(gxlib):
    """cuda:0 with the library's device state initialised."""
    import torch
    gxlib.check(gxlib.lib().gx_device_init(0), "gx_device_init")
    return torch.device("cuda:0")
