import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Parity tolerance against the fp32 oracle (the 2e-3 of the spec).
# fp32 tensors (states, fp32 outputs): max |x - y| / max |y| < REL_TOL.
# 16-bit outputs are checked element by element:
#     |x_i - y_i| <= REL_TOL * max|y| + U * |y_i|
# i.e. the same 2e-3 of the tensor's scale plus the rounding of x_i itself to
# its dtype: U is the unit roundoff (half an ulp, relative), 2^-8 for bf16
# (7 stored fraction bits) and 2^-11 for fp16 (10 bits). An fp32 result that
# meets 2e-3 meets this bound after rounding, whatever the element's size.
REL_TOL = 2e-3
ROUNDING = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}


def out_excess(x: torch.Tensor, y) -> float:
    """max_i |x_i - y_i| / (REL_TOL * max|y| + U * |y_i|): < 1 passes."""
    u = ROUNDING[x.dtype]
    xm = np.asarray(x.detach().float().cpu(), np.float64)
    ym = np.asarray(y.detach().float().cpu() if isinstance(y, torch.Tensor) else y, np.float64)
    scale = max(np.abs(ym).max(), 1e-30)
    bound = REL_TOL * scale * (1.0 + u) + u * np.abs(ym)
    return float((np.abs(xm - ym) / bound).max())


def assert_out_close(x: torch.Tensor, y, what="o"):
    """Output gate: element-wise 2e-3 of max|y| plus the dtype's own rounding
    of each element (fp32 outputs: plain max-relative 2e-3)."""
    if x.dtype == torch.float32:
        e = rel_err(x, y)
        assert e < REL_TOL, f"{what}: max rel err {e:.3e} >= {REL_TOL:.1e}"
        return
    q = out_excess(x, y)
    assert q < 1.0, (f"{what}: error reaches {q:.3f} of the element-wise bound "
                     f"(max rel err {rel_err(x, y):.3e})")


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
