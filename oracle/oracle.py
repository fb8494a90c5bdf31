"""TEST INFRASTRUCTURE ONLY: Python face of the C oracle (liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module; the product path (wkvm_b200) never imports it.

Functions take numpy float32 arrays in fla's [B, T, H, D] layout (or
[1, total, H, D] with cu_seqlens) and return (o, final_state) like fla's ops.
The arithmetic follows fla 0.5.1 token by token; see wkv_oracle.c for the
file:line citations.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "wkv_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", str(HERE), "liboracle.so"],
                       check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I = ctypes.c_int
        F = ctypes.c_float
        _lib.oracle_dplr.argtypes = [P] * 9 + [I] * 5 + [F, I]
        _lib.oracle_gdn.argtypes = [P] * 8 + [I] * 6 + [F, I, I]
    return _lib


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def default_threads() -> int:
    return int(os.environ.get("WKVM_ORACLE_THREADS", os.cpu_count() or 1))


def dplr_recurrence(r, w, k, v, a, b, scale=1.0, initial_state=None, cu_seqlens=None,
                    threads=None):
    """fp32 DPLR recurrence (fla fused_recurrent_rwkv7 semantics).

    r, w, k, a, b: [B, T, H, K]; v: [B, T, H, V]. Returns (o, h_final)."""
    r, w, k, v, a, b = map(_f32, (r, w, k, v, a, b))
    B, T, H, K = r.shape
    V = v.shape[-1]
    cu = None
    N = B
    if cu_seqlens is not None:
        cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int64))
        N = len(cu) - 1
    h = np.zeros((N, H, K, V), np.float32) if initial_state is None else _f32(initial_state).copy()
    o = np.zeros((B, T, H, V), np.float32)
    lib().oracle_dplr(_ptr(r), _ptr(w), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(o), _ptr(h),
                      _ptr(cu), N, T, H, K, V, float(scale), threads or default_threads())
    return o, h


def rwkv7_recurrence(r, w, k, v, kk, a_gate, scale=1.0, initial_state=None, cu_seqlens=None,
                     threads=None):
    """fla fused_mul_recurrent_rwkv7: a = -kk, b = kk * a_gate in fp32
    (fla/ops/rwkv7/fused_recurrent.py:94-96)."""
    kk = _f32(kk)
    a_gate = _f32(a_gate)
    return dplr_recurrence(r, w, k, v, -kk, kk * a_gate, scale, initial_state, cu_seqlens,
                           threads)


def gdn_recurrence(q, k, v, g, beta, scale=None, initial_state=None, cu_seqlens=None,
                   use_qk_l2norm=False, threads=None):
    """fp32 gated delta rule (fla fused_recurrent_gated_delta_rule semantics).

    q, k: [B, T, H, K]; v: [B, T, HV, V]; g, beta: [B, T, HV]."""
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if scale is None:
        scale = K ** -0.5
    cu = None
    N = B
    if cu_seqlens is not None:
        cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int64))
        N = len(cu) - 1
    h = np.zeros((N, HV, K, V), np.float32) if initial_state is None else _f32(initial_state).copy()
    o = np.zeros((B, T, HV, V), np.float32)
    lib().oracle_gdn(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(o), _ptr(h), _ptr(cu),
                     N, T, H, HV, K, V, float(scale), int(bool(use_qk_l2norm)),
                     threads or default_threads())
    return o, h
