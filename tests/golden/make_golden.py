"""Generates the golden vectors that pin the CPU oracle (tests/test_oracle.py).

wkvm keeps no golden vectors of its own and delegates its WKV arithmetic to
flash-linear-attention (fla) 0.5.1. This script imports fla's own fp32
torch reference functions — the ones fla tests its Triton kernels against —
and records inputs and outputs at small seeded shapes:

  fla/ops/generalized_delta_rule/dplr/naive.py:16  dplr_recurrence
  fla/ops/generalized_delta_rule/dplr/naive.py:41  dplr_chunkwise
  fla/ops/gated_delta_rule/naive.py:13             naive_recurrent_gated_delta_rule
  fla/ops/gated_delta_rule/naive.py:67             naive_chunk_gated_delta_rule

dplr_* force q * K^-0.5 (naive.py:23, :44); RWKV-7 calls with scale=1
(fla/layers/rwkv7.py:315,330), so r is pre-multiplied by sqrt(K) = 8 for
K = 64, which is exact in floating point.

Run once in a container where fla is importable:  python tests/golden/make_golden.py
Inputs are stored as bf16 bit patterns (uint16), outputs as float32.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from wkvm_b200 import synth  # noqa: E402


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def hf(t):  # [B, T, H, D] -> [B, H, T, D]
    return t.float().transpose(1, 2).contiguous()


def wkv7_case(name, B, T, H, N, seed, chunk=None):
    from fla.ops.generalized_delta_rule.dplr.naive import dplr_chunkwise, dplr_recurrence

    x = synth.rwkv7_inputs(B, T, H, N, seed=seed)
    r, w, k, v, kk, a = (x[n] for n in ("r", "w", "k", "v", "kk", "a"))
    alpha = -kk.float()
    beta = kk.float() * a.float()
    q = r.float() * (N ** 0.5)
    if chunk is None:
        o, ht = dplr_recurrence(hf(q), hf(k), hf(v), hf(alpha), hf(beta), hf(w),
                                initial_state=x["h0"].clone(), output_final_state=True)
    else:
        o, ht = dplr_chunkwise(hf(q), hf(k), hf(v), hf(alpha), hf(beta), hf(w),
                               initial_state=x["h0"].clone(), output_final_state=True,
                               chunk_size=chunk)
    out = {f"in_{n}": bf16_bits(x[n]) for n in ("r", "w", "k", "v", "kk", "a")}
    out["h0"] = x["h0"].numpy()
    out["o"] = o.float().transpose(1, 2).contiguous().numpy()
    out["ht"] = ht.float().numpy()
    np.savez_compressed(HERE / f"{name}.npz", **out)


def gdn_case(name, B, T, H, K, seed, chunk=None):
    from fla.ops.gated_delta_rule.naive import (naive_chunk_gated_delta_rule,
                                                naive_recurrent_gated_delta_rule)

    x = synth.gdn_inputs(B, T, H, K, seed=seed)
    args = [x[n].float() for n in ("q", "k", "v")]
    if chunk is None:
        o, ht = naive_recurrent_gated_delta_rule(*args, beta=x["beta"].float(),
                                                 g=x["g"].float(),
                                                 initial_state=x["h0"].clone(),
                                                 output_final_state=True)
    else:
        o, ht = naive_chunk_gated_delta_rule(*args, g=x["g"].float(), beta=x["beta"].float(),
                                             chunk_size=chunk, initial_state=x["h0"].clone(),
                                             output_final_state=True)
    out = {f"in_{n}": bf16_bits(x[n]) for n in ("q", "k", "v", "g", "beta")}
    out["h0"] = x["h0"].numpy()
    out["o"] = o.float().contiguous().numpy()
    out["ht"] = ht.float().numpy()
    np.savez_compressed(HERE / f"{name}.npz", **out)


def main():
    torch.manual_seed(0)
    wkv7_case("wkv7_recurrent_n64", B=2, T=32, H=2, N=64, seed=11)
    wkv7_case("wkv7_chunkwise_n64", B=1, T=128, H=2, N=64, seed=12, chunk=32)
    gdn_case("gdn_recurrent_k128", B=2, T=16, H=1, K=128, seed=13)
    gdn_case("gdn_chunk_k128", B=1, T=128, H=1, K=128, seed=14, chunk=64)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
