"""Prefill entry points (chunk_rwkv7 / chunk_gated_delta_rule and their
slot-native forms).

Sequences are run through the sm_100a kernels of libwkvm_b200.so; the
initial state comes from ``initial_state`` (or a bank slot) and the final
state goes to a new tensor (or back into the slot).
"""

from __future__ import annotations

import torch

from . import _lib
from . import ops as _ops


def chunk_dplr(r, w, k, v, a, b, scale, initial_state, output_final_state, cu_seqlens):
    return _ops._rwkv7_recurrent("wkvm_fused_recurrent_dplr", r, w, k, v, a, b, scale,
                                 initial_state, output_final_state, cu_seqlens)


def chunk_gdn(q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm,
              cu_seqlens):
    return _ops.fused_recurrent_gated_delta_rule(
        q, k, v, g=g, beta=beta, scale=scale, initial_state=initial_state,
        output_final_state=output_final_state, use_qk_l2norm_in_kernel=use_qk_l2norm,
        cu_seqlens=cu_seqlens)


def wkv7_prefill_slots(r, w, k, v, kk, a, bank_wkv, layer, slot_ids, cu_seqlens=None):
    if cu_seqlens is not None:
        raise NotImplementedError("varlen slot prefill: pass one row per sequence")
    return _ops.wkv7_decode_slots(r, w, k, v, kk, a, bank_wkv, layer, slot_ids)


def gdn_prefill_slots(q, k, v, g, beta, bank, layer, slot_ids, scale, use_qk_l2norm,
                      cu_seqlens=None):
    if cu_seqlens is not None:
        raise NotImplementedError("varlen slot prefill: pass one row per sequence")
    return _ops.gdn_decode_slots(q, k, v, g, beta, bank, layer, slot_ids, scale,
                                 use_qk_l2norm)


__all__ = ["chunk_dplr", "chunk_gdn", "wkv7_prefill_slots", "gdn_prefill_slots"]
_ = (_lib, torch)
