"""Parity at the benchmark configurations' full shapes, against the fp32
oracle (the recurrences of fla's fused_recurrent kernels):

* config 1: RWKV-7 slot decode, 256 of 1024 arena slots, L=24, H=32, N=64,
  64 steps of 24 overlapped launches. Every step: all 256 slots' outputs and
  a seeded subset of 8 slots' states (every layer) against the oracle
  stepped alongside; at the end: every output token and every active
  slot's final state (all layers), and the inactive slots untouched.
* config 2: RWKV-7 chunked prefill of B=16 x T=4096 x H=32 into arena
  slots: every output token and every final state.
* config 3: GDN decode over 512 slots (H=16, K=V=128, 64 steps), states of a
  subset every step and all outputs and final states; GDN chunked prefill of
  B=4 x T=8192 x H=16 into slots: every output token and every final state.

Gates: fp32 states max-relative 2e-3; bf16 outputs element-wise 2e-3 of the
tensor's scale plus bf16's rounding of each element (conftest)."""

import numpy as np
import pytest
import torch

from conftest import REL_TOL, assert_out_close, np32, rel_err
from oracle import oracle
from wkvm_b200 import ops, synth

pytestmark = pytest.mark.gpu

RW = ("r", "w", "k", "v", "kk", "a")
GD = ("q", "k", "v", "g", "beta")


def _arena(L, S, H, K, V, cuda, seed):
    bank = torch.empty(L, S + 1, H, K, V, device=cuda)
    bank.normal_(0.0, 0.1, generator=torch.Generator(device=cuda).manual_seed(seed))
    return bank


def _subset(ids, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(len(ids), generator=g)[:n].sort().values


def test_config1_decode_full_shape(cuda):
    L, S, H, N, B, steps = 24, 1024, 32, 64, 256, 64
    bank = _arena(L, S, H, N, N, cuda, seed=11)
    ids = synth.slot_ids(B, S + 1, seed=0).long()
    idle = torch.tensor(sorted(set(range(S + 1)) - set(ids.tolist())))
    idle_before = bank[:, idle[::16]].clone()
    h0 = bank[:, ids].clone()                                  # [L, B, H, N, N] on the device
    pos = _subset(ids, 8, seed=1)                              # batch rows checked every step
    sub = ids[pos]
    ids_dev = ops.slot_ids_tensor(ids, S + 1, cuda)
    # per layer, all steps at once: [B, steps, H, N]; step s reads [:, s:s+1]
    xs = [synth.rwkv7_inputs(B, steps, H, N, seed=500 + layer, device=cuda, state=False)
          for layer in range(L)]
    step_in = [[[xs[layer][n][:, s:s + 1].contiguous() for n in RW] for layer in range(L)]
               for s in range(steps)]
    outs = [[torch.empty(B, 1, H, N, dtype=torch.bfloat16, device=cuda) for _ in range(L)]
            for _ in range(steps)]
    h_sub = [np32(h0[layer, pos]) for layer in range(L)]
    x_sub = [{n: np32(xs[layer][n][pos]) for n in RW} for layer in range(L)]
    prev = ops.set_decode_overlap(True)
    try:
        for s in range(steps):
            for layer in range(L):
                ops.wkv7_decode_slots(*step_in[s][layer], bank, layer, ids_dev,
                                      out=outs[s][layer])
            torch.cuda.synchronize()
            got = bank[:, sub].cpu()
            for layer in range(L):
                ro, h_sub[layer] = oracle.rwkv7_recurrence(
                    *(x_sub[layer][n][:, s:s + 1] for n in RW), initial_state=h_sub[layer])
                e = rel_err(got[layer], h_sub[layer])
                assert e < REL_TOL, f"step {s} layer {layer}: state rel err {e:.2e}"
                assert_out_close(outs[s][layer][pos], ro, what=f"step {s} layer {layer}")
    finally:
        ops.set_decode_overlap(prev)
    ops.check_device_status(cuda)
    for layer in range(L):
        x = xs[layer]
        ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in RW),
                                         initial_state=np32(h0[layer]))
        o = torch.cat([outs[s][layer] for s in range(steps)], 1)
        assert_out_close(o, ro, what=f"layer {layer} outputs")
        assert rel_err(bank[layer, ids], rh) < REL_TOL, f"layer {layer} final states"
    assert torch.equal(bank[:, idle[::16]], idle_before)


def test_config2_prefill_full_shape(cuda):
    B, T, H, N, S = 16, 4096, 32, 64, 64
    bank = _arena(1, S, H, N, N, cuda, seed=12)
    ids = synth.slot_ids(B, S + 1, seed=2).long()
    h0 = bank[0, ids].clone()
    x = synth.rwkv7_inputs(B, T, H, N, seed=21, device=cuda, state=False)
    o = ops.wkv7_prefill_slots(*(x[n] for n in RW), bank, 0, ids)
    ops.check_device_status(cuda)
    for g0 in range(0, B, 4):  # the oracle runs four sequences at a time (host memory)
        rows = slice(g0, g0 + 4)
        ro, rh = oracle.rwkv7_recurrence(*(np32(x[n][rows]) for n in RW),
                                         initial_state=np32(h0[rows]))
        assert_out_close(o[rows], ro, what=f"sequences {g0}..{g0 + 3}")
        assert rel_err(bank[0, ids[rows]], rh) < REL_TOL


def test_config3_gdn_decode_full_shape(cuda):
    B, S, H, K, steps = 512, 1024, 16, 128, 64
    bank = _arena(1, S, H, K, K, cuda, seed=13)
    ids = synth.slot_ids(B, S + 1, seed=3).long()
    h0 = bank[0, ids].clone()
    pos = _subset(ids, 16, seed=4)
    sub = ids[pos]
    ids_dev = ops.slot_ids_tensor(ids, S + 1, cuda)
    x = synth.gdn_inputs(B, steps, H, K, seed=31, device=cuda, state=False)
    step_in = [[x[n][:, s:s + 1].contiguous() for n in GD] for s in range(steps)]
    outs = []
    h_sub = np32(h0[pos])
    x_sub = {n: np32(x[n][pos]) for n in GD}
    for s in range(steps):
        outs.append(ops.gdn_decode_slots(*step_in[s], bank, 0, ids_dev))
        ro, h_sub = oracle.gdn_recurrence(*(x_sub[n][:, s:s + 1] for n in GD),
                                          initial_state=h_sub)
        e = rel_err(bank[0, sub], h_sub)
        assert e < REL_TOL, f"step {s}: state rel err {e:.2e}"
        assert_out_close(outs[-1][pos], ro, what=f"step {s}")
    ops.check_device_status(cuda)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in GD), initial_state=np32(h0))
    assert_out_close(torch.cat(outs, 1), ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL


def test_config3_gdn_prefill_full_shape(cuda):
    B, T, H, K, S = 4, 8192, 16, 128, 16
    bank = _arena(1, S, H, K, K, cuda, seed=14)
    ids = synth.slot_ids(B, S + 1, seed=5).long()
    h0 = bank[0, ids].clone()
    x = synth.gdn_inputs(B, T, H, K, seed=41, device=cuda, state=False)
    o = ops.gdn_prefill_slots(*(x[n] for n in GD), bank, 0, ids)
    ops.check_device_status(cuda)
    for b in range(B):
        ro, rh = oracle.gdn_recurrence(*(np32(x[n][b:b + 1]) for n in GD),
                                       initial_state=np32(h0[b:b + 1]))
        assert_out_close(o[b:b + 1], ro, what=f"sequence {b}")
        assert rel_err(bank[0, ids[b:b + 1]], rh) < REL_TOL
