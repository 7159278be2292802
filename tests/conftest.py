import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def vg():
    import vibegemm_b200
    vibegemm_b200.lib()
    return vibegemm_b200


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle


def to_dev(a: np.ndarray):
    """uint16 fp16 bit patterns (host) -> float16 CUDA tensor."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)


def to_host(t) -> np.ndarray:
    """float16 tensor -> uint16 bit patterns (host)."""
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
