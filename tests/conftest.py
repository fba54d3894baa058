import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_PARENT = ROOT / "ucloud-ai-infra_b200"
for p in (str(ROOT), str(PKG_PARENT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    return np.load(GOLDEN / "golden.npz"), json.loads((GOLDEN / "golden.json").read_text())


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on a B200; fails loudly (no skip) when either is missing."""
    import torch

    from fp8_hand_b200 import _build, _native
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert torch.cuda.get_device_capability(0) == (10, 0), "GPU tests need sm_100 (B200)"
    _build.build()
    return _native.lib()
