"""Device-side slot id checks of the prefill, token-shift and fused time-mix
kernels: an id outside the arena (only possible in a device id tensor, which
the host does not check) is reported in the status word, the bad row is
skipped, and every other row gets exactly what a run without it gets."""

import pytest
import torch

from wkvm_b200 import ops, prefill, synth

pytestmark = pytest.mark.gpu


def _ids(lst, cuda):
    return torch.tensor(lst, dtype=torch.int32, device=cuda)


def _expect_slot_range(cuda):
    with pytest.raises(RuntimeError, match="SLOT_RANGE"):
        ops.check_device_status(cuda)
    ops.check_device_status(cuda)  # reset, clean again


def test_rwkv7_prefill_slots_bad_id(cuda):
    H, N, T = 2, 64, 130
    x = {k: v.to(cuda) for k, v in synth.rwkv7_inputs(3, T, H, N, seed=4, state=False).items()}
    bank = torch.randn(1, 5, H, N, N, device=cuda) * 0.1
    ref = bank.clone()
    args = [x[n] for n in ("r", "w", "k", "v", "kk", "a")]
    o = ops.wkv7_prefill_slots(*args, bank, 0, _ids([1, 9, 3], cuda))
    _expect_slot_range(cuda)
    keep = [0, 2]
    o_ref = ops.wkv7_prefill_slots(*(t[keep] for t in args), ref, 0, [1, 3])
    ops.check_device_status(cuda)
    assert torch.equal(bank, ref)
    assert torch.equal(o[keep], o_ref)


@pytest.mark.parametrize("limit", [2 << 30, 1, 0])  # two launches, windowed, one kernel
def test_gdn_prefill_slots_bad_id(cuda, monkeypatch, limit):
    monkeypatch.setattr(prefill, "GDN_WORKSPACE_LIMIT", limit)
    HV, K, T = 2, 128, 100
    x = {k: v.to(cuda) for k, v in synth.gdn_inputs(3, T, HV, K, seed=6, state=False).items()}
    bank = torch.randn(1, 5, HV, K, K, device=cuda) * 0.1
    ref = bank.clone()
    names = ("q", "k", "v", "g", "beta")
    o = prefill.gdn_prefill_slots(*(x[n] for n in names), bank, 0, _ids([2, 7, 4], cuda),
                                  K ** -0.5, False)
    _expect_slot_range(cuda)
    keep = [0, 2]
    o_ref = prefill.gdn_prefill_slots(*(x[n][keep] for n in names), ref, 0, [2, 4], K ** -0.5,
                                      False)
    ops.check_device_status(cuda)
    assert torch.equal(bank[0, [0, 1, 3]], ref[0, [0, 1, 3]])
    assert torch.equal(bank[0, [2, 4]], ref[0, [2, 4]])
    assert torch.equal(o[keep], o_ref)


def test_shift_mix_bad_id(cuda):
    D, S = 128, 6
    shift = torch.randn(S, D, device=cuda).to(torch.bfloat16)
    ref = shift.clone()
    x = torch.randn(3, 1, D, device=cuda).to(torch.bfloat16)
    mix = [torch.rand(D, device=cuda).to(torch.bfloat16) for _ in range(2)]
    outs = ops.wkv7_shift_mix_slots(x, mix, shift, _ids([1, 11, 4], cuda))
    _expect_slot_range(cuda)
    ref_outs = ops.wkv7_shift_mix_slots(x[[0, 2]], mix, ref, [1, 4])
    ops.check_device_status(cuda)
    assert torch.equal(shift, ref)
    for o, r in zip(outs, ref_outs):
        assert torch.equal(o[[0, 2]], r)


def test_timemix_bad_id(cuda):
    B, H, N = 3, 2, 64
    D = H * N
    mk = lambda *s, sc=1.0: (torch.randn(*s, device=cuda) * sc).to(torch.bfloat16)
    acts = [mk(B, D) for _ in range(6)]  # r, w_raw, k, v, a_raw, g
    prm = [mk(D, sc=0.5), mk(D, sc=0.5), mk(H, N, sc=0.5), mk(D, sc=0.3), mk(D, sc=0.1)]
    bank = torch.randn(1, 5, H, N, N, device=cuda) * 0.1
    ref = bank.clone()
    r, w, k, v, a, g = acts
    o = ops.wkv7_timemix_decode_slots(r, w, k, v, None, None, a, g, *prm, 64e-5, bank, 0,
                                      _ids([3, 8, 1], cuda))
    _expect_slot_range(cuda)
    keep = [0, 2]
    o_ref = ops.wkv7_timemix_decode_slots(*(t[keep] for t in (r, w, k, v)), None, None,
                                          a[keep], g[keep], *prm, 64e-5, ref, 0, [3, 1])
    ops.check_device_status(cuda)
    assert torch.equal(bank, ref)
    assert torch.equal(o[keep], o_ref)


def test_debug_checks_raise_at_the_call(cuda):
    """With ops.set_debug_checks(True) a device id tensor with a duplicate
    is rejected before the launch, and a device-side error raises from the
    op that met it instead of waiting for check_device_status."""
    H, N = 2, 64
    x = {k: v.to(cuda) for k, v in synth.rwkv7_inputs(3, 1, H, N, seed=7, state=False).items()}
    bank = torch.randn(1, 6, H, N, N, device=cuda) * 0.1
    args = [x[n] for n in ("r", "w", "k", "v", "kk", "a")]
    prev = ops.set_debug_checks(True)
    try:
        with pytest.raises(RuntimeError, match="DUPLICATE"):
            ops.wkv7_decode_slots(*args, bank, 0, _ids([1, 4, 1], cuda))
        with pytest.raises(RuntimeError, match="SLOT_RANGE"):
            ops.wkv7_decode_slots(*args, bank, 0, _ids([1, 4, 9], cuda))
        ops.wkv7_decode_slots(*args, bank, 0, _ids([1, 4, 5], cuda))
    finally:
        ops.set_debug_checks(prev)
    ops.check_device_status(cuda)


def test_gdn_prefill_reports_records_beyond_fp16(cuda, monkeypatch):
    """The two-launch GDN prefill keeps its per-chunk records in fp16. Values
    too large for fp16 (here |v| ~ 1e5) are reported in the status word as
    WKVM_ERR_UNSUPPORTED instead of flowing on as infinities; the one-kernel
    path (no workspace, tf32 operands) handles the same call."""
    from conftest import REL_TOL, assert_out_close, np32, rel_err
    from oracle import oracle
    HV, K, T = 2, 128, 200
    x = synth.gdn_inputs(1, T, HV, K, seed=6)
    x["v"] = (x["v"].float() * 1e5).to(torch.bfloat16)
    d = {k: v.to(cuda) for k, v in x.items()}
    names = ("q", "k", "v", "g", "beta")
    ops.check_device_status(cuda)
    ops.chunk_gated_delta_rule(*(d[n] for n in names), initial_state=d["h0"],
                               output_final_state=True)
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        ops.check_device_status(cuda)
    monkeypatch.setattr(prefill, "GDN_WORKSPACE_LIMIT", 0)
    o, ht = ops.chunk_gated_delta_rule(*(d[n] for n in names), initial_state=d["h0"],
                                       output_final_state=True)
    ops.check_device_status(cuda)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in names), initial_state=np32(x["h0"]))
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL
