import random
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tt-cadlab_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"
SEED = 213919  # the reference's test seed (tests/conftest.py:12)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libpalu_b200.so")
    config.addinivalue_line("markers", "slow: long-running CPU oracle comparisons")


@pytest.fixture(autouse=True)
def reset_seeds():
    torch.manual_seed(SEED)
    np.random.seed(SEED)
    random.seed(SEED)


def load_golden(name: str) -> dict:
    z = np.load(GOLDEN / f"{name}.npz")
    return {k: torch.from_numpy(z[k]) if z[k].dtype != np.uint8 else z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from palu_b200 import build
    build.build()
    return torch.device("cuda:0")
