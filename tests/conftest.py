import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long-running")


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load_golden(name):
    import int8_kernel_lab_b200 as m

    data = np.load(GOLDEN / f"{name}.npz")
    shape = m.ConvShape(*[int(v) for v in data["shape"]])
    return shape, data["x"], data["w"], data["b"], data["y"]


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    assert major == 10, "GPU tests need an sm_100 device"
    return torch
