"""Host-side logic of the op wrappers (CPU only, no kernel launches)."""

import pytest
import torch

from wkvm_b200 import ops
from wkvm_b200._lib import WkvmError
from wkvm_b200.state import RWKV7StateLayout


def test_slot_id_validation_range_and_duplicates():
    with pytest.raises(WkvmError, match="SLOT_RANGE"):
        ops.slot_ids_tensor([1, 9], 5, "cpu")
    with pytest.raises(WkvmError, match="SLOT_RANGE"):
        ops.slot_ids_tensor([-1], 5, "cpu")
    with pytest.raises(WkvmError, match="DUPLICATE"):
        ops.slot_ids_tensor([2, 3, 2], 5, "cpu")
    t = ops.slot_ids_tensor([0, 4, 1], 5, "cpu")
    assert t.dtype == torch.int32 and t.tolist() == [0, 4, 1]
    assert ops.slot_ids_tensor([], 5, "cpu").numel() == 0


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(1, 1, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.fused_mul_recurrent_rwkv7(x, x, x, x, x, x)
    with pytest.raises(ValueError, match="CUDA"):
        ops.fused_recurrent_gated_delta_rule(x, x, x, g=x[..., 0], beta=x[..., 0])


def test_fla_argument_errors():
    x = torch.zeros(2, 3, 1, 64)
    with pytest.raises(DeprecationWarning):
        ops.fused_mul_recurrent_rwkv7(x, x, x, x, x, x, head_first=True)
    with pytest.raises(ValueError, match="batch size is expected to be 1"):
        ops.fused_mul_recurrent_rwkv7(x, x, x, x, x, x, cu_seqlens=torch.tensor([0, 3]))
    y = torch.zeros(1, 6, 1, 64)
    with pytest.raises(ValueError, match="number of initial states"):
        ops.fused_mul_recurrent_rwkv7(y, y, y, y, y, y, initial_state=torch.zeros(3, 1, 64, 64),
                                      cu_seqlens=torch.tensor([0, 3, 6]))
    with pytest.raises(NotImplementedError):
        ops.fused_recurrent_gated_delta_rule(x, x, x, gk=x)
    with pytest.raises(ValueError, match="same number of heads"):
        ops.chunk_gated_delta_rule(x, torch.zeros(2, 3, 2, 64), x, x[..., 0], x[..., 0])


def test_family_geometry_matches_reference_layout():
    lay = RWKV7StateLayout(n_layer=3, hidden_size=64, num_heads=2, head_dim=32, head_v_dim=32)
    wkv = torch.zeros(lay.n_layer, 5, *lay.wkv_shape)
    shift = torch.zeros(lay.n_layer, 2, 5, lay.hidden_size, dtype=torch.bfloat16)
    outer, ostr, sstr, row, ns = ops._family_geometry(wkv, 1)
    assert (outer, ns, row) == (3, 5, 2 * 32 * 32 * 4) and ostr == 5 * row and sstr == row
    outer, ostr, sstr, row, ns = ops._family_geometry(shift, 2)
    assert (outer, ns, row) == (6, 5, 128) and ostr == 5 * 128
    assert lay.wkv_bytes_per_slot() == 3 * 2 * 32 * 32 * 4


def test_slot_affine_rejects_chained_pairs():
    fam = torch.zeros(2, 6, 4)
    # slot 2 is pair 0's destination and pair 1's source: pairs run at once
    with pytest.raises(ValueError, match="another pair's source"):
        ops.slot_affine(fam, 1, [2, 3], [1, 2], None, 0.5)
    with pytest.raises(ValueError, match="another pair's source"):
        ops.slot_affine(fam, 1, [4, 5], [1, 2], [5, 3], 0.5, 0.5)


def test_debug_checks_toggle():
    from wkvm_b200 import _lib
    prev = ops.set_debug_checks(True)
    try:
        assert _lib.post_call is not None
    finally:
        ops.set_debug_checks(prev)
    assert (_lib.post_call is None) == (not prev)
