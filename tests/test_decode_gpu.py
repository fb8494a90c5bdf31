"""Parity of the recurrent / decode kernels against the CPU oracle
(fla fused_recurrent semantics). Tolerance: max-relative 2e-3 (REL_TOL)."""

import numpy as np
import pytest
import torch

from conftest import REL_TOL, assert_out_close, np32, rel_err
from oracle import oracle
from wkvm_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _to(x, dev):
    return {k: v.to(dev) for k, v in x.items()}


@pytest.mark.parametrize("N", [32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("T", [1, 7])
def test_fused_mul_recurrent_rwkv7(cuda, N, dtype, T):
    B, H = 3, 4
    x = synth.rwkv7_inputs(B, T, H, N, seed=N + T, dtype=dtype)
    d = _to(x, cuda)
    o, ht = ops.fused_mul_recurrent_rwkv7(d["r"], d["w"], d["k"], d["v"], d["kk"], d["a"],
                                          scale=1.0, initial_state=d["h0"],
                                          output_final_state=True)
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in ("r", "w", "k", "v", "kk", "a")),
                                     initial_state=np32(x["h0"]))
    assert o.dtype == dtype and ht.dtype == torch.float32
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_no_initial_state_and_no_final_state(cuda):
    x = synth.rwkv7_inputs(2, 3, 2, 64, seed=5)
    d = _to(x, cuda)
    o, ht = ops.fused_mul_recurrent_rwkv7(d["r"], d["w"], d["k"], d["v"], d["kk"], d["a"])
    assert ht is None
    ro, _ = oracle.rwkv7_recurrence(*(np32(x[n]) for n in ("r", "w", "k", "v", "kk", "a")))
    assert_out_close(o, ro)


def test_dplr_general_form_and_scale(cuda):
    x = synth.rwkv7_inputs(2, 5, 3, 64, seed=9)
    d = _to(x, cuda)
    a = -d["kk"]
    b = (d["kk"].float() * d["a"].float()).to(torch.bfloat16)
    o, ht = ops.fused_recurrent_rwkv7(d["r"], d["w"], d["k"], d["v"], a, b,
                                      initial_state=d["h0"])
    ro, rh = oracle.dplr_recurrence(np32(x["r"]), np32(x["w"]), np32(x["k"]), np32(x["v"]),
                                    np32(a), np32(b), scale=64 ** -0.5,
                                    initial_state=np32(x["h0"]))
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_varlen_cu_seqlens(cuda):
    lens = [3, 0, 11, 1]
    H, N = 2, 64
    tot = sum(lens)
    x = synth.rwkv7_inputs(1, tot, H, N, seed=4, num_states=len(lens))
    d = _to(x, cuda)
    cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int64)
    o, ht = ops.fused_mul_recurrent_rwkv7(d["r"], d["w"], d["k"], d["v"], d["kk"], d["a"],
                                          initial_state=d["h0"], output_final_state=True,
                                          cu_seqlens=cu.to(cuda))
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in ("r", "w", "k", "v", "kk", "a")),
                                     initial_state=np32(x["h0"]), cu_seqlens=cu.numpy())
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL
    assert torch.equal(ht[1], d["h0"][1])  # empty sequence: state passes through


def _bank(L, S, H, N, dev, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(L, S, H, N, N, generator=g) * 0.1).to(dev)


def test_decode_slots_in_place_and_neighbours_untouched(cuda):
    L, S, H, N, B = 2, 9, 4, 64, 4
    bank = _bank(L, S, H, N, cuda)
    before = bank.clone()
    ids = [7, 2, 5, 8]
    x = synth.rwkv7_inputs(B, 1, H, N, seed=3, state=False)
    d = _to(x, cuda)
    o = ops.wkv7_decode_slots(d["r"], d["w"], d["k"], d["v"], d["kk"], d["a"], bank, 1, ids)
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in ("r", "w", "k", "v", "kk", "a")),
                                     initial_state=np32(before[1, ids]))
    assert_out_close(o, ro)
    assert rel_err(bank[1, ids], rh) < REL_TOL
    untouched = [s for s in range(S) if s not in ids]
    assert torch.equal(bank[1, untouched], before[1, untouched])
    assert torch.equal(bank[0], before[0])  # other layer
    ops.check_device_status(cuda)


def test_decode_slots_4096_steps(cuda):
    """North-star gate: outputs and final states within 2e-3 after 4096
    recurrent steps (bf16 I/O, fp32 state)."""
    L, S, H, N, B, steps = 1, 6, 4, 64, 3, 4096
    bank = _bank(L, S, H, N, cuda, seed=1)
    ids = [4, 1, 3]
    h_ref = np32(bank[0, ids])
    x = synth.rwkv7_inputs(B, steps, H, N, seed=21, state=False)
    d = _to(x, cuda)
    ids_dev = ops.slot_ids_tensor(ids, S, cuda)
    outs = []
    for t in range(steps):
        outs.append(ops.wkv7_decode_slots(*(d[n][:, t:t + 1] for n in ("r", "w", "k", "v", "kk", "a")),
                                          bank, 0, ids_dev))
    o = torch.cat(outs, 1)
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in ("r", "w", "k", "v", "kk", "a")),
                                     initial_state=h_ref)
    assert_out_close(o, ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL
    # the whole 4096-token sequence in one multi-token call agrees as well
    bank2 = _bank(L, S, H, N, cuda, seed=1)
    o2 = ops.wkv7_decode_slots(*(d[n] for n in ("r", "w", "k", "v", "kk", "a")), bank2, 0, ids)
    assert_out_close(o2, ro)
    assert rel_err(bank2[0, ids], rh) < REL_TOL


def test_decode_slots_bad_id_reports_and_skips(cuda):
    bank = _bank(1, 4, 2, 64, cuda)
    before = bank.clone()
    x = _to(synth.rwkv7_inputs(1, 1, 2, 64, seed=2, state=False), cuda)
    bad = torch.tensor([9], dtype=torch.int32, device=cuda)  # device ids are not host-checked
    ops.wkv7_decode_slots(x["r"], x["w"], x["k"], x["v"], x["kk"], x["a"], bank, 0, bad)
    with pytest.raises(RuntimeError, match="SLOT_RANGE"):
        ops.check_device_status(cuda)
    assert torch.equal(bank, before)
    ops.check_device_status(cuda)  # reset and clean again


@pytest.mark.parametrize("K", [64, 128])
@pytest.mark.parametrize("HV_mult", [1, 2])
@pytest.mark.parametrize("l2", [False, True])
def test_gdn_recurrent(cuda, K, HV_mult, l2):
    B, T, H = 2, 5, 2
    x = synth.gdn_inputs(B, T, H, K, HV=H * HV_mult, seed=K + HV_mult)
    if l2:  # un-normalised q, k exercise the in-kernel normalisation
        x["q"] = (x["q"].float() * 3.0).to(torch.bfloat16)
        x["k"] = (x["k"].float() * 0.5).to(torch.bfloat16)
    d = _to(x, cuda)
    o, ht = ops.fused_recurrent_gated_delta_rule(d["q"], d["k"], d["v"], g=d["g"], beta=d["beta"],
                                                 initial_state=d["h0"], output_final_state=True,
                                                 use_qk_l2norm_in_kernel=l2)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in ("q", "k", "v", "g", "beta")),
                                   initial_state=np32(x["h0"]), use_qk_l2norm=l2)
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_gdn_decode_slots_long(cuda):
    S, HV, K, B, steps = 5, 2, 128, 2, 1024
    g = torch.Generator().manual_seed(3)
    bank = (torch.randn(1, S, HV, K, K, generator=g) * 0.1).to(cuda)
    ids = [3, 1]
    h_ref = np32(bank[0, ids])
    x = synth.gdn_inputs(B, steps, HV, K, seed=8, state=False)
    d = _to(x, cuda)
    ids_dev = ops.slot_ids_tensor(ids, S, cuda)
    outs = [ops.gdn_decode_slots(*(d[n][:, t:t + 1] for n in ("q", "k", "v", "g", "beta")),
                                 bank, 0, ids_dev) for t in range(steps)]
    o = torch.cat(outs, 1)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in ("q", "k", "v", "g", "beta")),
                                   initial_state=h_ref)
    assert_out_close(o, ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL


@pytest.mark.parametrize("L", [2, 12])
@pytest.mark.parametrize("graphed", [True, False])
def test_decode_overlap_layer_loop(cuda, L, graphed):
    """Overlapped (programmatic dependent launch) decode over a layer loop at
    the config-0 shape (B=8, H=12, N=64; L=12, and L=2 where the same layer
    comes back every other launch), 64 steps launched back to back: either
    all 64 x L launches captured in one CUDA graph (no gaps between
    launches, the case where short launches could pile up) or eagerly.
    Every step's output and the final state match the oracle run layer by
    layer."""
    S, H, N, B, steps = 40, 12, 64, 8, 64
    bank = _bank(L, S, H, N, cuda, seed=4)
    slot_list = synth.slot_ids(B, S, seed=3).long()
    h_ref = [np32(bank[layer, slot_list]) for layer in range(L)]
    ids = ops.slot_ids_tensor(slot_list, S, cuda)
    names = ("r", "w", "k", "v", "kk", "a")
    # per layer, all steps drawn at once as [B, steps, H, N]; step s is [:, s:s+1]
    xs = [synth.rwkv7_inputs(B, steps, H, N, seed=1000 + layer, state=False) for layer in range(L)]
    ds = [_to(x, cuda) for x in xs]
    step_in = [[[ds[layer][n][:, s:s + 1].contiguous() for n in names] for layer in range(L)]
               for s in range(steps)]
    outs = [[torch.empty(B, 1, H, N, dtype=torch.bfloat16, device=cuda) for _ in range(L)]
            for _ in range(steps)]

    def run():
        for s in range(steps):
            for layer in range(L):
                ops.wkv7_decode_slots(*step_in[s][layer], bank, layer, ids, out=outs[s][layer])

    ops.status_word(cuda)
    prev = ops.set_decode_overlap(True)
    try:
        if graphed:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                run()
            bank[:, slot_list] = torch.from_numpy(np.stack(h_ref, 0)).to(cuda)
            torch.cuda.synchronize()
            graph.replay()
        else:
            run()
        torch.cuda.synchronize()
    finally:
        ops.set_decode_overlap(prev)
    for layer in range(L):
        x = xs[layer]
        ro, h = oracle.rwkv7_recurrence(*(np32(x[n]) for n in names), initial_state=h_ref[layer])
        o = torch.cat([outs[s][layer] for s in range(steps)], 1)
        assert_out_close(o, ro, what=f"layer {layer}")
        assert rel_err(bank[layer, slot_list], h) < REL_TOL
    ops.check_device_status(cuda)
