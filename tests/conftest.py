import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Parity tolerance against the fp32 oracle: max |x - y| / max |y| over the
# tensor. fp32 tensors (states, fp32 outputs) must meet REL_TOL itself. A
# bf16/fp16 output additionally carries its own rounding (a bf16 value is
# within 2^-8 of the fp32 value it rounds, relative to that value), so its
# bound is REL_TOL + that rounding, and its mean error must meet REL_TOL.
REL_TOL = 2e-3
ROUNDING = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}


def out_tol(t: torch.Tensor) -> float:
    return REL_TOL + ROUNDING[t.dtype]


def assert_out_close(x: torch.Tensor, y, what="o"):
    """Output gate: max-relative within out_tol(x), mean-relative within REL_TOL."""
    e = rel_err(x, y)
    assert e < out_tol(x), f"{what}: max rel err {e:.3e} >= {out_tol(x):.3e}"
    xm = np.asarray(x.detach().float().cpu(), np.float64)
    ym = np.asarray(y.detach().float().cpu() if isinstance(y, torch.Tensor) else y, np.float64)
    m = np.abs(xm - ym).mean() / max(np.abs(ym).mean(), 1e-30)
    assert m < REL_TOL, f"{what}: mean rel err {m:.3e}"


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
