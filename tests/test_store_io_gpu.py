"""Batched asynchronous hibernation (WARM tier) and the COLD round trip on
the GPU: hibernate slots while decode keeps writing other slots, persist the
batch in wkvm's file format, load it back and wake it into other slots;
every copy is bit-exact."""

import pytest
import torch

from wkvm_b200 import ops, store_io, synth
from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

pytestmark = pytest.mark.gpu


def test_hibernate_persist_wake_bit_exact(cuda, tmp_path):
    lay = RWKV7StateLayout(n_layer=3, hidden_size=128, num_heads=2, head_dim=64, head_v_dim=64)
    bank = RWKV7StateBank(lay, num_slots=16, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    bank.wkv.normal_(0.0, 0.1, generator=g)
    bank.shift.copy_(torch.randn(bank.shift.shape, device=cuda, generator=g))
    sess = [3, 9, 1, 12, 6]
    before_wkv = bank.wkv[:, sess].clone()
    before_shift = bank.shift[:, :, sess].clone()
    batch = store_io.hibernate(bank, sess)
    # decode of other slots continues meanwhile
    x = synth.rwkv7_inputs(2, 1, 2, 64, seed=1, device=cuda, state=False)
    for layer in range(3):
        ops.wkv7_decode_slots(x["r"], x["w"], x["k"], x["v"], x["kk"], x["a"], bank.wkv, layer,
                              [2, 4])
    batch.wait()
    assert batch.nbytes == 5 * (lay.wkv_bytes_per_slot() + lay.shift_bytes_per_slot())
    for i in range(len(sess)):
        t = batch.tensors(i)
        assert t["wkv"].shape == (3, 2, 64, 64) and t["shift"].shape == (3, 2, 128)
        assert torch.equal(t["wkv"], before_wkv[:, i].cpu())
        assert torch.equal(t["shift"], before_shift[:, :, i].cpu())

    fp = store_io.fingerprint(lay)
    recs = [store_io.Record(name=f"s{s}", version=0, fingerprint=fp, num_computed_tokens=4,
                            token_ids=(1, 2, 3, 4, 5)) for s in sess]
    paths = store_io.persist_many(tmp_path, recs, batch, threads=3)
    index, cold = store_io.read_index(tmp_path)
    assert cold == {r.handle for r in recs} and set(index) == cold
    assert [p.name for p in paths] == [f"s{s}_v0.safetensors" for s in sess]

    # wake: the hibernated batch into fresh slots (one kernel per family), and
    # the COLD files into others (one per session)
    warm_slots, cold_slots = [13, 14, 15, 10, 11], [5, 7, 8, 2, 4]
    store_io.wake(bank, warm_slots, batch)
    store_io.wake(bank, cold_slots, [store_io.load_cold(p) for p in paths])
    ops.check_device_status(cuda)
    torch.cuda.synchronize()
    for slots in (warm_slots, cold_slots):
        assert torch.equal(bank.wkv[:, slots], before_wkv)
        assert torch.equal(bank.shift[:, :, slots], before_shift)


def test_hibernate_into_reused_buffers(cuda):
    lay = RWKV7StateLayout(n_layer=2, hidden_size=64, num_heads=1, head_dim=64, head_v_dim=64)
    bank = RWKV7StateBank(lay, num_slots=8, device=cuda)
    bank.wkv.normal_(0.0, 0.1, generator=torch.Generator(device=cuda).manual_seed(2))
    pool = store_io.pinned_buffers(bank, 4)
    for sess in ([1, 5, 2], [7, 3]):
        b = store_io.hibernate(bank, sess, pool).wait()
        assert b.wkv.data_ptr() == pool[0].data_ptr()
        assert torch.equal(b.wkv, bank.wkv[:, sess].transpose(0, 1).cpu())
    with pytest.raises(ValueError):
        store_io.hibernate(bank, [1, 2, 3, 4, 5], pool)


def test_wake_from_pageable_host_tensors(cuda):
    """wake() given plain (unpinned) CPU tensors stages each one in pinned
    memory; every staged copy must outlive the restore that reads it, so
    several sessions woken in a row all land bit-exact."""
    lay = RWKV7StateLayout(n_layer=4, hidden_size=128, num_heads=2, head_dim=64, head_v_dim=64)
    bank = RWKV7StateBank(lay, num_slots=16, device=cuda)
    g = torch.Generator().manual_seed(11)
    sessions = [{"wkv": torch.randn(4, 2, 64, 64, generator=g),
                 "shift": torch.randn(4, 2, 128, generator=g).to(lay.dtype)} for _ in range(8)]
    assert not sessions[0]["wkv"].is_pinned()
    slots = [9, 2, 14, 5, 11, 3, 7, 16]
    store_io.wake(bank, slots, sessions)
    # whatever the host allocator hands out next must not disturb the result
    junk = [torch.full((4, 2, 64, 64), 7.0).pin_memory() for _ in range(8)]
    torch.cuda.synchronize()
    for s, t in zip(slots, sessions):
        assert torch.equal(bank.wkv[:, s].cpu(), t["wkv"])
        assert torch.equal(bank.shift[:, :, s].cpu(), t["shift"])
    del junk
