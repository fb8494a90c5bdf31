"""Parity against the reference's own GPU implementation: fla 0.5.1's Triton
kernels (the ones wkvm's RWKV-7 model runs), on identical seeded inputs.
Skipped when fla or Triton cannot run on the box.

fla's recurrent kernels compute in fp32 like ours, so states agree to fp32
rounding. fla's chunk kernels use bf16 tensor-core dots (the state is cast to
bf16 inside the state pass), so against them the bound is looser; both are
checked against the fp32 oracle elsewhere."""

import pytest
import torch

from conftest import REL_TOL, assert_out_close, rel_err
from wkvm_b200 import ops, synth

pytestmark = pytest.mark.gpu

fla_rwkv7 = pytest.importorskip("fla.ops.rwkv7")
fla_gdn = pytest.importorskip("fla.ops.gated_delta_rule")


def test_decode_matches_fla_triton(cuda):
    x = synth.rwkv7_inputs(16, 1, 8, 64, seed=1, device=cuda)
    args = [x[n] for n in ("r", "w", "k", "v", "kk", "a")]
    o1, h1 = fla_rwkv7.fused_mul_recurrent_rwkv7(*args, scale=1.0, initial_state=x["h0"],
                                                 output_final_state=True)
    o2, h2 = ops.fused_mul_recurrent_rwkv7(*args, scale=1.0, initial_state=x["h0"],
                                           output_final_state=True)
    assert rel_err(h2, h1) < 1e-5
    assert_out_close(o2, o1.float())


def test_multistep_matches_fla_triton(cuda):
    x = synth.rwkv7_inputs(4, 40, 4, 64, seed=2, device=cuda)
    args = [x[n] for n in ("r", "w", "k", "v", "kk", "a")]
    o1, h1 = fla_rwkv7.fused_mul_recurrent_rwkv7(*args, scale=1.0, initial_state=x["h0"],
                                                 output_final_state=True)
    o2, h2 = ops.fused_mul_recurrent_rwkv7(*args, scale=1.0, initial_state=x["h0"],
                                           output_final_state=True)
    assert rel_err(h2, h1) < 1e-4
    assert_out_close(o2, o1.float())


def test_chunk_close_to_fla_triton(cuda):
    x = synth.rwkv7_inputs(2, 256, 4, 64, seed=3, device=cuda)
    a = -x["kk"]
    b = (x["kk"].float() * x["a"].float()).to(torch.bfloat16)
    c = [x["r"], x["w"], x["k"], x["v"], a, b]
    o1, h1 = fla_rwkv7.chunk_rwkv7(*c, scale=1.0, initial_state=x["h0"], output_final_state=True,
                                   safe_gate=True, chunk_size=64)
    o2, h2 = ops.chunk_rwkv7(*c, scale=1.0, initial_state=x["h0"], output_final_state=True)
    # fla rounds its chunk operands to bf16; 1e-2 covers that difference.
    assert rel_err(h2, h1) < 1e-2
    assert rel_err(o2, o1) < 1e-2


def test_gdn_decode_matches_fla_triton(cuda):
    g = synth.gdn_inputs(32, 1, 4, 128, seed=4, device=cuda)
    o1, h1 = fla_gdn.fused_recurrent_gated_delta_rule(g["q"], g["k"], g["v"], g["g"], beta=g["beta"],
                                                      initial_state=g["h0"],
                                                      output_final_state=True)
    o2, h2 = ops.fused_recurrent_gated_delta_rule(g["q"], g["k"], g["v"], g["g"], beta=g["beta"],
                                                  initial_state=g["h0"], output_final_state=True)
    assert rel_err(h2, h1) < 1e-5
    assert_out_close(o2, o1.float())


def test_gdn_chunk_close_to_fla_triton(cuda):
    g = synth.gdn_inputs(2, 256, 2, 128, seed=5, device=cuda)
    o1, h1 = fla_gdn.chunk_gated_delta_rule(g["q"], g["k"], g["v"], g["g"], g["beta"],
                                            initial_state=g["h0"], output_final_state=True)
    o2, h2 = ops.chunk_gated_delta_rule(g["q"], g["k"], g["v"], g["g"], g["beta"],
                                        initial_state=g["h0"], output_final_state=True)
    assert rel_err(h2, h1) < 2e-2
    assert rel_err(o2, o1) < 2e-2
    _ = REL_TOL
