"""Seeded synthetic inputs with the value distributions of the benchmark
configurations (there is no public dataset for this path).

RWKV-7 (the op-level distribution of the decode/prefill configs):
  r, k, v ~ N(0, 1); log-decay w = -0.6065306597 * sigmoid(x), x ~ N(0, 1)
  (fla/layers/rwkv7.py:271); kk = normalize(k') per head, k' ~ N(0, 1);
  a_gate = sigmoid(y), y ~ N(0, 1); all cast to the activation dtype;
  fp32 state h0 ~ N(0, 0.1^2).
GDN: q, k L2-normalised N(0, 1); v ~ N(0, 1); g = -softplus(N(0, 1));
  beta = sigmoid(N(0, 1)).
Tensors are drawn in a fixed order from one generator per call.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

W_SCALE = -0.6065306597126334


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def rwkv7_inputs(B, T, H, N, *, seed=0, dtype=torch.bfloat16, device="cpu", state=True,
                 num_states=None):
    """Returns dict r, w, k, v, kk, a (a = sigmoid gate), each [B, T, H, N],
    and h0 [num_states or B, H, N, N] fp32 when ``state``."""
    g = _gen(seed, device)
    shape = (B, T, H, N)

    def randn(*s):
        return torch.randn(*s, generator=g, device=device, dtype=torch.float32)

    out = {
        "r": randn(*shape).to(dtype),
        "w": (W_SCALE * torch.sigmoid(randn(*shape))).to(dtype),
        "k": randn(*shape).to(dtype),
        "v": randn(*shape).to(dtype),
        "kk": F.normalize(randn(*shape), dim=-1).to(dtype),
        "a": torch.sigmoid(randn(*shape)).to(dtype),
    }
    if state:
        out["h0"] = randn(num_states or B, H, N, N) * 0.1
    return out


def gdn_inputs(B, T, H, K, V=None, HV=None, *, seed=0, dtype=torch.bfloat16, device="cpu",
               state=True, num_states=None):
    """Returns dict q, k [B,T,H,K]; v [B,T,HV,V]; g, beta [B,T,HV]; h0."""
    V = V or K
    HV = HV or H
    g = _gen(seed, device)

    def randn(*s):
        return torch.randn(*s, generator=g, device=device, dtype=torch.float32)

    out = {
        "q": F.normalize(randn(B, T, H, K), dim=-1).to(dtype),
        "k": F.normalize(randn(B, T, H, K), dim=-1).to(dtype),
        "v": randn(B, T, HV, V).to(dtype),
        "g": (-F.softplus(randn(B, T, HV))).to(dtype),
        "beta": torch.sigmoid(randn(B, T, HV)).to(dtype),
    }
    if state:
        out["h0"] = randn(num_states or B, HV, K, V) * 0.1
    return out


def slot_ids(n, num_slots, *, seed=0) -> torch.Tensor:
    """n distinct slot ids drawn without replacement from 1..num_slots-1
    (slot 0 is wkvm's reserved padding row), int32, CPU."""
    g = _gen(seed, "cpu")
    perm = torch.randperm(num_slots - 1, generator=g)[:n] + 1
    return perm.to(torch.int32)
