"""Pins the tcgen05 layer (descriptors, TMEM layout) with one tf32 GEMM tile."""

import pytest
import torch

from wkvm_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _tf32(x):
    b = x.view(torch.int32)
    return ((b + 0x1000) & ~0x1FFF).view(torch.float32)


@pytest.mark.parametrize("N", [64, 128])
@pytest.mark.parametrize("a_in_tmem", [0, 1])
def test_tf32_tile_matches_fp64(cuda, N, a_in_tmem):
    g = torch.Generator().manual_seed(N)
    A = _tf32(torch.randn(128, 64, generator=g)).to(cuda)
    B = _tf32(torch.randn(N, 64, generator=g)).to(cuda)
    D = torch.full((128, N), float("nan"), device=cuda)
    _lib.call("wkvm_selftest_tf32_mma", A.data_ptr(), B.data_ptr(), D.data_ptr(), N, a_in_tmem,
              ops.status_word(cuda).data_ptr(), torch.cuda.current_stream().cuda_stream)
    ops.check_device_status(cuda)
    ref = (A.double() @ B.double().T)
    # tf32-exact operands: only fp32 accumulation error remains
    err = (D.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err
