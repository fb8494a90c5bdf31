"""Chunked tensor-core prefill vs the fp32 oracle recurrence
(fla chunk_rwkv7 semantics; the chunk form reassociates the same recurrence)."""

import numpy as np
import pytest
import torch

from conftest import REL_TOL, assert_out_close, np32, rel_err
from oracle import oracle
from wkvm_b200 import ops, prefill, synth

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "kk", "a")


def _to(x, dev):
    return {k: v.to(dev) for k, v in x.items()}


def _ab(d):
    a = -d["kk"]
    b = (d["kk"].float() * d["a"].float()).to(d["kk"].dtype)
    return a, b


@pytest.mark.parametrize("T", [1, 63, 64, 200])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("h0", [True, False])
def test_chunk_rwkv7_matches_oracle(cuda, T, dtype, h0):
    B, H, N = 2, 3, 64
    x = synth.rwkv7_inputs(B, T, H, N, seed=T, dtype=dtype)
    d = _to(x, cuda)
    a, b = _ab(d)
    o, ht = ops.chunk_rwkv7(d["r"], d["w"], d["k"], d["v"], a, b, scale=1.0,
                            initial_state=d["h0"] if h0 else None, output_final_state=True,
                            safe_gate=True, chunk_size=64)
    ro, rh = oracle.dplr_recurrence(np32(d["r"]), np32(d["w"]), np32(d["k"]), np32(d["v"]),
                                    np32(a), np32(b), initial_state=np32(x["h0"]) if h0 else None)
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_chunk_rwkv7_4096_tokens(cuda):
    """North-star gate at 4096 tokens: o and final state within 2e-3."""
    B, T, H, N = 2, 4096, 2, 64
    x = synth.rwkv7_inputs(B, T, H, N, seed=77)
    d = _to(x, cuda)
    a, b = _ab(d)
    o, ht = ops.chunk_rwkv7(d["r"], d["w"], d["k"], d["v"], a, b, scale=1.0,
                            initial_state=d["h0"], output_final_state=True)
    ro, rh = oracle.dplr_recurrence(np32(d["r"]), np32(d["w"]), np32(d["k"]), np32(d["v"]),
                                    np32(a), np32(b), initial_state=np32(x["h0"]))
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_prefill_slots_in_place(cuda):
    L, S, H, N, B, T = 2, 7, 2, 64, 3, 130
    g = torch.Generator().manual_seed(5)
    bank = (torch.randn(L, S, H, N, N, generator=g) * 0.1).to(cuda)
    before = bank.clone()
    ids = [5, 1, 6]
    x = synth.rwkv7_inputs(B, T, H, N, seed=6, state=False)
    d = _to(x, cuda)
    o = ops.wkv7_prefill_slots(*(d[n] for n in NAMES), bank, 1, ids)
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in NAMES), initial_state=np32(before[1, ids]))
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(bank[1, ids], rh) < REL_TOL
    rest = [s for s in range(S) if s not in ids]
    assert torch.equal(bank[1, rest], before[1, rest]) and torch.equal(bank[0], before[0])


def test_prefill_slots_varlen(cuda):
    S, H, N = 6, 2, 64
    lens = [70, 0, 5, 128]
    ids = [2, 4, 1, 5]
    g = torch.Generator().manual_seed(9)
    bank = (torch.randn(1, S, H, N, N, generator=g) * 0.1).to(cuda)
    before = bank.clone()
    x = synth.rwkv7_inputs(1, sum(lens), H, N, seed=10, state=False)
    d = _to(x, cuda)
    cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int64)
    o = ops.wkv7_prefill_slots(*(d[n] for n in NAMES), bank, 0, ids, cu_seqlens=cu.to(cuda))
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in NAMES),
                                     initial_state=np32(before[0, ids]), cu_seqlens=cu.numpy())
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL
    assert torch.equal(bank[0, 4], before[0, 4])  # the empty sequence's slot


def test_prefill_then_decode_matches_one_recurrence(cuda):
    """prefill(T) followed by decode steps equals the oracle over T + steps."""
    S, H, N, B, T, steps = 4, 2, 64, 2, 96, 5
    bank = torch.zeros(1, S, H, N, N, device=cuda)
    ids = [3, 1]
    x = synth.rwkv7_inputs(B, T + steps, H, N, seed=12, state=False)
    d = _to(x, cuda)
    o1 = ops.wkv7_prefill_slots(*(d[n][:, :T] for n in NAMES), bank, 0, ids)
    outs = [ops.wkv7_decode_slots(*(d[n][:, T + i:T + i + 1] for n in NAMES), bank, 0, ids)
            for i in range(steps)]
    o = torch.cat([o1] + outs, 1)
    ro, rh = oracle.rwkv7_recurrence(*(np32(x[n]) for n in NAMES))
    assert_out_close(o, ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL


def test_other_head_dims_use_recurrent_path(cuda):
    x = synth.rwkv7_inputs(2, 70, 2, 32, seed=3)
    d = _to(x, cuda)
    a, b = _ab(d)
    o, ht = ops.chunk_rwkv7(d["r"], d["w"], d["k"], d["v"], a, b, initial_state=d["h0"],
                            output_final_state=True)
    ro, rh = oracle.dplr_recurrence(np32(d["r"]), np32(d["w"]), np32(d["k"]), np32(d["v"]),
                                    np32(a), np32(b), initial_state=np32(x["h0"]))
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


GDN = ("q", "k", "v", "g", "beta")


@pytest.fixture(params=["two_phase", "windowed", "one_kernel"])
def gdn_path(request, monkeypatch):
    """GDN prefill path: two launches over a full workspace, the same with a
    one-chunk window (state carried between windows), or the fused kernel."""
    limit = {"two_phase": prefill.GDN_WORKSPACE_LIMIT, "windowed": 1, "one_kernel": 0}
    monkeypatch.setattr(prefill, "GDN_WORKSPACE_LIMIT", limit[request.param])
    return request.param


@pytest.mark.parametrize("T", [1, 100, 200])
@pytest.mark.parametrize("hv_mult", [1, 2])
@pytest.mark.parametrize("l2", [False, True])
def test_chunk_gdn_matches_oracle(cuda, gdn_path, T, hv_mult, l2):
    B, H, K = 2, 2, 128
    x = synth.gdn_inputs(B, T, H, K, HV=H * hv_mult, seed=T + hv_mult)
    if l2:
        x["q"] = (x["q"].float() * 2.5).to(torch.bfloat16)
        x["k"] = (x["k"].float() * 0.7).to(torch.bfloat16)
    d = _to(x, cuda)
    o, ht = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                       initial_state=d["h0"], output_final_state=True,
                                       use_qk_l2norm_in_kernel=l2)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in GDN), initial_state=np32(x["h0"]),
                                   use_qk_l2norm=l2)
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_chunk_gdn_fp16_inputs(cuda, gdn_path):
    # fp16 runs the Gram block on fp16 operands (kind::f16, both operands fp16)
    B, T, H, K = 2, 200, 2, 128
    x = synth.gdn_inputs(B, T, H, K, HV=4, seed=12, dtype=torch.float16)
    d = _to(x, cuda)
    o, ht = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                       initial_state=d["h0"], output_final_state=True,
                                       use_qk_l2norm_in_kernel=True)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in GDN), initial_state=np32(x["h0"]),
                                   use_qk_l2norm=True)
    ops.check_device_status(cuda)
    assert o.dtype == torch.float16
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_chunk_gdn_4096_tokens(cuda, gdn_path):
    B, T, H, K = 1, 4096, 2, 128
    x = synth.gdn_inputs(B, T, H, K, seed=31)
    d = _to(x, cuda)
    o, ht = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                       initial_state=d["h0"], output_final_state=True)
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in GDN), initial_state=np32(x["h0"]))
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_gdn_prefill_slots_varlen(cuda, gdn_path):
    S, HV, K = 6, 2, 128
    lens = [70, 0, 130]
    ids = [4, 2, 5]
    g = torch.Generator().manual_seed(2)
    bank = (torch.randn(1, S, HV, K, K, generator=g) * 0.1).to(cuda)
    before = bank.clone()
    x = synth.gdn_inputs(1, sum(lens), HV, K, seed=3, state=False)
    d = _to(x, cuda)
    cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int64)
    o = ops.gdn_prefill_slots(*(d[n] for n in GDN), bank, 0, ids, cu_seqlens=cu.to(cuda))
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in GDN), initial_state=np32(before[0, ids]),
                                   cu_seqlens=cu.numpy())
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(bank[0, ids], rh) < REL_TOL
    rest = [0, 1, 3]
    assert torch.equal(bank[0, rest], before[0, rest]) and torch.equal(bank[0, 2], before[0, 2])


def test_chunk_rwkv7_varlen_cu_seqlens(cuda):
    lens = [130, 0, 64, 7]
    H, N = 2, 64
    x = synth.rwkv7_inputs(1, sum(lens), H, N, seed=41, num_states=len(lens))
    d = _to(x, cuda)
    a, b = _ab(d)
    cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int64)
    o, ht = ops.chunk_rwkv7(d["r"], d["w"], d["k"], d["v"], a, b, scale=1.0,
                            initial_state=d["h0"], output_final_state=True,
                            cu_seqlens=cu.to(cuda))
    ro, rh = oracle.dplr_recurrence(np32(d["r"]), np32(d["w"]), np32(d["k"]), np32(d["v"]),
                                    np32(a), np32(b), initial_state=np32(x["h0"]),
                                    cu_seqlens=cu.numpy())
    ops.check_device_status(cuda)
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL
    assert torch.equal(ht[1], d["h0"][1])


@pytest.mark.parametrize("limit", [2 << 30, 0])  # two launches, one kernel
def test_chunk_gdn_fp32_gates_stay_on_16bit_path(cuda, monkeypatch, limit):
    """16-bit q/k/v with fp32 g and beta (what fla's GDN layers pass) runs the
    16-bit chunk kernels: with gates that bf16 represents exactly the result
    is bit-identical to the all-bf16 call (the recurrent fallback would round
    differently), and gates that bf16 cannot hold match the oracle."""
    monkeypatch.setattr(prefill, "GDN_WORKSPACE_LIMIT", limit)
    B, T, H, K = 2, 200, 2, 128
    x = synth.gdn_inputs(B, T, H, K, seed=12)
    d = _to(x, cuda)
    args = dict(scale=K ** -0.5, initial_state=d["h0"], output_final_state=True)
    o16, h16 = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], **args)
    o32, h32 = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"].float(),
                                          d["beta"].float(), **args)
    assert torch.equal(o16, o32) and torch.equal(h16, h32)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=torch.Generator().manual_seed(3)))
    beta = torch.rand(B, T, H, generator=torch.Generator().manual_seed(4))
    o, ht = ops.chunk_gated_delta_rule(d["q"], d["k"], d["v"], g.to(cuda), beta.to(cuda), **args)
    ro, rh = oracle.gdn_recurrence(np32(x["q"]), np32(x["k"]), np32(x["v"]), g.numpy(),
                                   beta.numpy(), initial_state=np32(x["h0"]))
    ops.check_device_status(cuda)
    assert o.dtype == torch.bfloat16
    assert_out_close(o, ro)
    assert rel_err(ht, rh) < REL_TOL


def test_gdn_decode_fp32_gates(cuda):
    B, H, K = 3, 2, 128
    x = synth.gdn_inputs(B, 1, H, K, seed=13)
    d = _to(x, cuda)
    bank = torch.zeros(1, 5, H, K, K, device=cuda)
    bank[0, [1, 2, 4]] = d["h0"]
    o = ops.gdn_decode_slots(d["q"], d["k"], d["v"], d["g"].float(), d["beta"].float(), bank, 0,
                             [1, 2, 4])
    ro, rh = oracle.gdn_recurrence(*(np32(x[n]) for n in ("q", "k", "v", "g", "beta")),
                                   initial_state=np32(x["h0"]))
    assert o.dtype == torch.bfloat16
    assert_out_close(o, ro)
    assert rel_err(bank[0, [1, 2, 4]], rh) < REL_TOL
