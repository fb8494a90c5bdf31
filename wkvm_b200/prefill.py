"""Prefill entry points (chunk_rwkv7 / chunk_gated_delta_rule and their
slot-native forms).

RWKV-7 (head dim 64) runs a fused chunked tensor-core kernel (tcgen05 tf32,
64-token chunks, state kept on chip across chunks). The GDN sibling
(K = V = 128) runs two launches over a device workspace: a chunk-parallel WY
kernel, then a sequential pass with the state resident in tensor memory
(or, with the workspace switched off, one fused kernel). Other head sizes run
the recurrent kernel, which streams the state once and loops over tokens.
The initial state comes from ``initial_state`` (or a bank slot) and the final
state goes to a new tensor (or back into the slot).
"""

from __future__ import annotations

import torch

from . import _lib
from . import ops as _ops

# Upper bound on the GDN prefill workspace (bytes). Past it the chunks are
# processed in windows; 0 selects the one-kernel path.
GDN_WORKSPACE_LIMIT = 2 << 30


def _gdn_workspace(nseq, T, HV, K, V, device):
    """Device workspace for the two-launch GDN prefill, or None."""
    limit = GDN_WORKSPACE_LIMIT
    if limit <= 0:
        return None
    lib = _lib.load()
    full = lib.wkvm_gdn_chunk_workspace_bytes(nseq, T, HV, K, V)
    if full <= 0:
        return None
    # one window: carried state + one chunk record per (sequence, head)
    minimum = nseq * HV * K * V * 4 + 256 + lib.wkvm_gdn_chunk_workspace_bytes(nseq, 1, HV, K, V)
    size = full if full <= limit else max(limit, minimum)
    return torch.empty(size, dtype=torch.uint8, device=device)



def chunk_dplr(r, w, k, v, a, b, scale, initial_state, output_final_state, cu_seqlens):
    """fla chunk_dplr_delta_rule semantics; returns (o, final_state or None)."""
    return _ops._rwkv7_recurrent("wkvm_chunk_dplr", r, w, k, v, a, b, scale, initial_state,
                                 output_final_state, cu_seqlens)


def chunk_gdn(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm,
              cu_seqlens):
    """fla chunk_gated_delta_rule semantics; returns (o, final_state or None)."""
    _ops._require_cuda(q, k, v, g, beta, initial_state)
    (q, k, v, g, beta), dt = _ops._gdn_acts(q, k, v, g, beta)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    cu = _ops._cu(cu_seqlens, q.device)
    h0 = _ops._state(initial_state)
    o = torch.empty_like(v)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=q.device) if output_final_state else None
    ws = _gdn_workspace(N, T, HV, K, V, q.device)
    with torch.cuda.device(q.device):
        _lib.call("wkvm_chunk_gated_delta_rule", _ops._ptr(q), _ops._ptr(k), _ops._ptr(v),
                  _ops._ptr(g), _ops._ptr(beta), _ops._ptr(o), _ops._ptr(h0), _ops._ptr(ht),
                  _ops._ptr(cu), N if cu is not None else B, T, H, HV, K, V, float(scale),
                  int(bool(use_qk_l2norm)), dt, _ops._ptr(ws), ws.numel() if ws is not None else 0,
                  _ops._ptr(_ops.status_word(q.device)), _ops._stream(q.device))
    return o, ht


def wkv7_prefill_slots(r, w, k, v, kk, a, bank_wkv, layer, slot_ids, cu_seqlens=None,
                       out=None):
    """RWKV-7 prefill with initial and final state in bank_wkv[layer, slot_ids].
    Inputs [B, T, H, N] (or [1, total, H, N] with cu_seqlens); returns o."""
    _ops._require_cuda(r, w, k, v, kk, a, bank_wkv)
    layer_t = _ops._bank_layer(bank_wkv, layer)
    (r, w, k, v, kk, a), dt = _ops._acts(r, w, k, v, kk, a)
    B, T, H, K = r.shape
    V = v.shape[-1]
    if tuple(layer_t.shape[1:]) != (H, K, V):
        raise ValueError("bank layer shape does not match H, K, V")
    _ops._check_varlen(r, None, cu_seqlens)
    nseq = B if cu_seqlens is None else len(cu_seqlens) - 1
    ids = _ops.slot_ids_tensor(slot_ids, layer_t.shape[0], r.device)
    if ids.numel() != nseq:
        raise ValueError(f"{ids.numel()} slot ids for {nseq} sequences")
    cu = _ops._cu(cu_seqlens, r.device)
    o = torch.empty_like(v) if out is None else out
    with torch.cuda.device(r.device):
        _lib.call("wkvm_wkv7_prefill_slots", _ops._ptr(r), _ops._ptr(w), _ops._ptr(k),
                  _ops._ptr(v), _ops._ptr(kk), _ops._ptr(a), _ops._ptr(o), _ops._ptr(layer_t),
                  layer_t.shape[0], _ops._ptr(ids), _ops._ptr(cu), nseq, T, H, K, V, dt,
                  _ops._ptr(_ops.status_word(r.device)), _ops._stream(r.device))
    return o


def gdn_prefill_slots(q, k, v, g, beta, bank, layer, slot_ids, scale, use_qk_l2norm,
                      cu_seqlens=None, out=None):
    """Chunked GDN prefill with initial and final state in bank[layer, slot_ids]."""
    _ops._require_cuda(q, k, v, g, beta, bank)
    layer_t = _ops._bank_layer(bank, layer)
    (q, k, v, g, beta), dt = _ops._gdn_acts(q, k, v, g, beta)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if tuple(layer_t.shape[1:]) != (HV, K, V):
        raise ValueError("bank layer shape does not match HV, K, V")
    _ops._check_varlen(q, None, cu_seqlens)
    nseq = B if cu_seqlens is None else len(cu_seqlens) - 1
    ids = _ops.slot_ids_tensor(slot_ids, layer_t.shape[0], q.device)
    if ids.numel() != nseq:
        raise ValueError(f"{ids.numel()} slot ids for {nseq} sequences")
    cu = _ops._cu(cu_seqlens, q.device)
    o = torch.empty_like(v) if out is None else out
    ws = _gdn_workspace(nseq, T, HV, K, V, q.device)
    with torch.cuda.device(q.device):
        _lib.call("wkvm_gdn_prefill_slots", _ops._ptr(q), _ops._ptr(k), _ops._ptr(v),
                  _ops._ptr(g), _ops._ptr(beta), _ops._ptr(o), _ops._ptr(layer_t),
                  layer_t.shape[0], _ops._ptr(ids), _ops._ptr(cu), nseq, T, H, HV, K, V,
                  float(scale), int(bool(use_qk_l2norm)), dt, _ops._ptr(ws),
                  ws.numel() if ws is not None else 0,
                  _ops._ptr(_ops.status_word(q.device)), _ops._stream(q.device))
    return o
