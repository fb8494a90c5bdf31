"""wkvm_b200: B200-native (sm_100a) state-slot hot path of wkvm.

RWKV-7 WKV and gated-delta-rule recurrences over fp32 per-request state
slots — decode in place by slot id, chunked prefill into slots, and slot
fork / snapshot / restore / migrate — behind fla's operator signatures and
wkvm's state-bank interface. All compute runs in libwkvm_b200.so.
"""

from . import ops
from .ops import (
    chunk_gated_delta_rule,
    chunk_rwkv7,
    fused_mul_recurrent_rwkv7,
    fused_recurrent_gated_delta_rule,
    fused_recurrent_rwkv7,
    gdn_decode_slots,
    gdn_prefill_slots,
    wkv7_decode_slots,
    wkv7_prefill_slots,
)

__all__ = [
    "ops",
    "chunk_gated_delta_rule",
    "chunk_rwkv7",
    "fused_mul_recurrent_rwkv7",
    "fused_recurrent_gated_delta_rule",
    "fused_recurrent_rwkv7",
    "gdn_decode_slots",
    "gdn_prefill_slots",
    "wkv7_decode_slots",
    "wkv7_prefill_slots",
]
