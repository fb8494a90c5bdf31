"""Slot fork / zero / snapshot / restore are bit-exact; the bank keeps
wkvm's RWKV7StateBank semantics (wkvm tests/test_rwkv7_gpu.py:72-120)."""

import pytest
import torch

from wkvm_b200 import ops
from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

pytestmark = pytest.mark.gpu

LAYOUT = RWKV7StateLayout(n_layer=3, hidden_size=64, num_heads=2, head_dim=32, head_v_dim=32,
                          dtype=torch.bfloat16)


def _bank(cuda, fill=True):
    b = RWKV7StateBank(LAYOUT, num_slots=4, device=cuda)
    if fill:
        b.wkv.normal_()
        b.shift.normal_()
    return b


def test_zero_slots(cuda):
    bank = _bank(cuda)
    before_w, before_s = bank.wkv.clone(), bank.shift.clone()
    bank.zero_slots({"wkv": 2, "shift": 3})
    assert bank.wkv[:, 2].abs().sum().item() == 0
    assert bank.shift[:, :, 3].abs().sum().item() == 0
    keep = [0, 1, 3, 4]
    assert torch.equal(bank.wkv[:, keep], before_w[:, keep])
    keep = [0, 1, 2, 4]
    assert torch.equal(bank.shift[:, :, keep], before_s[:, :, keep])


def test_fork_bit_exact(cuda):
    bank = _bank(cuda)
    before_w, before_s = bank.wkv.clone(), bank.shift.clone()
    bank.fork([{"wkv": 1, "shift": 1}, {"wkv": 2, "shift": 2}],
              [{"wkv": 4, "shift": 3}, {"wkv": 3, "shift": 4}])
    assert torch.equal(bank.wkv[:, 4], before_w[:, 1]) and torch.equal(bank.wkv[:, 3], before_w[:, 2])
    assert torch.equal(bank.shift[:, :, 3], before_s[:, :, 1])
    assert torch.equal(bank.shift[:, :, 4], before_s[:, :, 2])
    assert torch.equal(bank.wkv[:, :3], before_w[:, :3])
    with pytest.raises(ValueError, match="overlap"):
        bank.fork([{"wkv": 1, "shift": 1}], [{"wkv": 1, "shift": 2}])


def test_snapshot_restore_bit_exact_reference_layout(cuda):
    bank = _bank(cuda)
    snap = bank.snapshot({"wkv": 2, "shift": 2})
    # identical to wkvm StateStore.save's host tensors (wkvm/store.py:130-131)
    assert snap["wkv"].is_pinned() and snap["wkv"].shape == (3, 2, 32, 32)
    assert torch.equal(snap["wkv"], bank.wkv[:, 2].cpu())
    assert torch.equal(snap["shift"], bank.shift[:, :, 2].cpu())
    bank.zero_slots({"wkv": 4, "shift": 4})
    bank.restore({"wkv": 4, "shift": 4}, snap)
    assert torch.equal(bank.wkv[:, 4], bank.wkv[:, 2])
    assert torch.equal(bank.shift[:, :, 4], bank.shift[:, :, 2])


def test_snapshot_many_large_rows(cuda):
    # rows larger than one 16 KiB stripe and a ragged last stripe
    fam = torch.randn(5, 7, 3, 1000, device=cuda)  # row = 12000 B
    ids = [6, 0, 3]
    out = ops.slot_snapshot(fam, 1, ids)
    torch.cuda.synchronize()
    assert torch.equal(out, fam[:, ids].permute(1, 0, 2, 3).cpu())
    fam2 = torch.zeros_like(fam)
    ops.slot_restore(fam2, 1, ids, out)
    assert torch.equal(fam2[:, ids], fam[:, ids])
    assert fam2[:, [1, 2, 4, 5]].abs().sum().item() == 0


def test_empty_batches_are_noops(cuda):
    bank = _bank(cuda)
    before = bank.wkv.clone()
    ops.slot_zero(bank.wkv, 1, [])
    ops.slot_copy(bank.wkv, 1, [], [])
    assert torch.equal(bank.wkv, before)


def test_device_ids_out_of_range_report(cuda):
    bank = _bank(cuda)
    before = bank.wkv.clone()
    bad = torch.tensor([7], dtype=torch.int32, device=cuda)
    ops.slot_zero(bank.wkv, 1, bad)
    with pytest.raises(RuntimeError, match="SLOT_RANGE"):
        ops.check_device_status(cuda)
    assert torch.equal(bank.wkv, before)


def test_migrate_same_device_path(cuda):
    """The migrate kernel on one GPU (src and dst banks both local): the
    multi-GPU case differs only in the destination pointer."""
    a, b = _bank(cuda), _bank(cuda, fill=False)
    a.migrate_to(b, [{"wkv": 1, "shift": 2}], [{"wkv": 3, "shift": 4}]).synchronize()
    assert torch.equal(b.wkv[:, 3], a.wkv[:, 1])
    assert torch.equal(b.shift[:, :, 4], a.shift[:, :, 2])
    assert b.wkv[:, [0, 1, 2, 4]].abs().sum().item() == 0


def test_bank_packer_round_trip(cuda):
    """The device packer used for cross-process migration: rows of both
    families for n slots -> one flat buffer -> another bank, bit-exact."""
    from wkvm_b200 import shard
    a, b = _bank(cuda), _bank(cuda, fill=False)
    pack, _, _ = shard.bank_packer(a)
    _, unpack, empty = shard.bank_packer(b)
    buf = pack([2, 4])
    assert buf.numel() == empty(2).numel()
    unpack([1, 3], buf)
    torch.cuda.synchronize()
    assert torch.equal(b.wkv[:, 1], a.wkv[:, 2]) and torch.equal(b.wkv[:, 3], a.wkv[:, 4])
    assert torch.equal(b.shift[:, :, 1], a.shift[:, :, 2])
    assert torch.equal(b.shift[:, :, 3], a.shift[:, :, 4])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_migrate_between_gpus_peer_stores(cuda):
    a = _bank(torch.device("cuda", 0))
    b = RWKV7StateBank(LAYOUT, num_slots=4, device=torch.device("cuda", 1))
    with torch.cuda.device(0):
        ev = a.migrate_to(b, [{"wkv": 2, "shift": 3}], [{"wkv": 4, "shift": 1}])
        ev.synchronize()
    torch.cuda.synchronize(1)
    assert torch.equal(b.wkv[:, 4].cpu(), a.wkv[:, 2].cpu())
    assert torch.equal(b.shift[:, :, 1].cpu(), a.shift[:, :, 3].cpu())
    assert b.wkv[:, [0, 1, 2, 3]].abs().sum().item() == 0


def test_mutation_rules_bit_exact(cuda):
    """decay and merge on live slots equal wkvm's StateStore rules computed
    by torch on the host copies (wkvm/store.py:260-268, 298-305)."""
    bank = _bank(cuda)
    w0, s0 = bank.wkv.cpu(), bank.shift.cpu()
    bank.decay({"wkv": 2, "shift": 2}, alpha=0.9)
    assert torch.equal(bank.wkv[:, 2].cpu(), (w0[:, 2].float() * 0.9).to(torch.float32))
    assert torch.equal(bank.shift.cpu(), s0)
    bank.merge({"wkv": 4, "shift": 4}, {"wkv": 1, "shift": 1}, {"wkv": 3, "shift": 3}, weight=0.3)
    ref_w = ((1.0 - 0.3) * w0[:, 1].float() + 0.3 * w0[:, 3].float()).to(torch.float32)
    ref_s = ((1.0 - 0.3) * s0[:, :, 1].float() + 0.3 * s0[:, :, 3].float()).to(torch.bfloat16)
    assert torch.equal(bank.wkv[:, 4].cpu(), ref_w)
    assert torch.equal(bank.shift[:, :, 4].cpu(), ref_s)
    ops.check_device_status(cuda)
