"""Pins the CPU oracle against golden vectors from fla's own fp32 reference
functions (tests/golden/make_golden.py) and checks its host-side properties.
CPU only."""

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import oracle

GOLD = Path(__file__).resolve().parent / "golden"


def _bf16(bits: np.ndarray) -> np.ndarray:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).float().numpy()


def _load(name):
    z = np.load(GOLD / f"{name}.npz")
    return {k: (_bf16(z[k]) if k.startswith("in_") else z[k]) for k in z.files}


@pytest.mark.parametrize("name", ["wkv7_recurrent_n64", "wkv7_chunkwise_n64"])
def test_oracle_matches_fla_dplr(name):
    g = _load(name)
    o, ht = oracle.rwkv7_recurrence(g["in_r"], g["in_w"], g["in_k"], g["in_v"], g["in_kk"],
                                    g["in_a"], scale=1.0, initial_state=g["h0"])
    # recurrence vs recurrence: fp32 rounding only; vs fla's chunkwise form:
    # reassociated fp32 sums over 128 tokens.
    tol = 1e-5 if "recurrent" in name else 1e-4
    assert rel_err(o, g["o"]) < tol
    assert rel_err(ht, g["ht"]) < tol


@pytest.mark.parametrize("name", ["gdn_recurrent_k128", "gdn_chunk_k128"])
def test_oracle_matches_fla_gdn(name):
    g = _load(name)
    o, ht = oracle.gdn_recurrence(g["in_q"], g["in_k"], g["in_v"], g["in_g"], g["in_beta"],
                                  initial_state=g["h0"])
    tol = 1e-5 if "recurrent" in name else 1e-4
    assert rel_err(o, g["o"]) < tol
    assert rel_err(ht, g["ht"]) < tol


def test_oracle_varlen_equals_separate():
    rng = np.random.default_rng(0)
    H, N = 2, 32
    lens = [5, 0, 9]
    tot = sum(lens)
    x = {n: rng.standard_normal((1, tot, H, N)).astype(np.float32) for n in "rwkvab"}
    x["w"] = -0.6 * (1 / (1 + np.exp(-x["w"])))
    h0 = rng.standard_normal((3, H, N, N)).astype(np.float32) * 0.1
    cu = np.cumsum([0] + lens)
    o, ht = oracle.dplr_recurrence(x["r"], x["w"], x["k"], x["v"], x["a"], x["b"],
                                   initial_state=h0, cu_seqlens=cu)
    for i, (s, e) in enumerate(zip(cu[:-1], cu[1:])):
        oi, hi = oracle.dplr_recurrence(*(x[n][:, s:e] for n in "rwkvab"),
                                        initial_state=h0[i:i + 1])
        np.testing.assert_array_equal(o[:, s:e], oi)
        np.testing.assert_array_equal(ht[i:i + 1], hi)
    # a zero-length sequence leaves its state untouched
    np.testing.assert_array_equal(ht[1], h0[1])


def test_oracle_threads_deterministic():
    rng = np.random.default_rng(1)
    x = {n: rng.standard_normal((3, 7, 4, 64)).astype(np.float32) for n in "rwkvab"}
    o1, h1 = oracle.dplr_recurrence(*(x[n] for n in "rwkvab"), threads=1)
    o8, h8 = oracle.dplr_recurrence(*(x[n] for n in "rwkvab"), threads=8)
    np.testing.assert_array_equal(o1, o8)
    np.testing.assert_array_equal(h1, h8)


def test_gdn_l2norm_equals_prenormalised():
    rng = np.random.default_rng(2)
    B, T, H, K = 2, 6, 2, 64
    q = rng.standard_normal((B, T, H, K)).astype(np.float32)
    k = rng.standard_normal((B, T, H, K)).astype(np.float32)
    v = rng.standard_normal((B, T, H, K)).astype(np.float32)
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    o1, h1 = oracle.gdn_recurrence(q, k, v, g, beta, use_qk_l2norm=True)
    qn = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
    kn = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    o2, h2 = oracle.gdn_recurrence(qn, kn, v, g, beta)
    assert rel_err(o1, o2) < 1e-5 and rel_err(h1, h2) < 1e-5
