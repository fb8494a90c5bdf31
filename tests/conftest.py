import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Parity tolerance for outputs and final states against the fp32 oracle:
# max |x - y| / max |y| over the tensor (bf16 I/O, fp32 state).
REL_TOL = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def rel_err(x, y) -> float:
    x = np.asarray(x.detach().float().cpu() if isinstance(x, torch.Tensor) else x, np.float64)
    y = np.asarray(y.detach().float().cpu() if isinstance(y, torch.Tensor) else y, np.float64)
    denom = max(np.abs(y).max(), 1e-30)
    return float(np.abs(x - y).max() / denom)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from wkvm_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
